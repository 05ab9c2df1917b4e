"""Host-side sequence dispatch over GPUs (one process per GPU).

Decode sequences are independent, so the multi-GPU path shards them: every
rank holds a full weight replica and its own KV pool, and no collective runs
on the data path. This module decides which rank serves which sequence and
what happens when a rank fails:

  plan_shards   longest-first greedy placement by KV tokens (prompt + output)
                onto the least-loaded rank; sequences that share a cached
                prefix (`prefix_id`) are placed together, so the prefix is
                prefilled once per rank and restored from a device snapshot
                (the engine's prefix cache, `src/chat/engine.rs:516-601`). A
                prefix group heavier than the mean per-rank load is cut into
                the fewest pieces of at most that load (one prefix prefill per
                piece) instead of overloading one rank. The plan is a pure
                function of its inputs: every rank computes the same one
                locally, no broadcast needed.
  requeue       the same placement rule applied to the sequences of failed
                ranks, over the surviving ranks only; sequences already placed
                on survivors stay where they are.
  run_with_failover
                runs one rank's shard and reports through a key-value store
                (torch.distributed TCPStore): `done/<rank>` with its results,
                or `fail/<rank>` when its work raised. A rank that has neither
                reported nor failed by the deadline counts as failed too (it
                never joined, died, or is too slow). The deadline runs from
                one start time shared by all ranks, and the first rank to
                decide writes the failed set once (compare_set): every rank
                uses that set. Survivors requeue the failed ranks' sequences,
                serve their share, publish `requeued/<rank>`, and every rank
                still running returns the merged results of all sequences.
                Failure is learned on the host between steps: no device wait
                depends on another rank.
"""

from __future__ import annotations

import json
import time
from dataclasses import dataclass
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple


@dataclass(frozen=True)
class SeqRequest:
    seq_id: int
    prompt_len: int
    output_len: int
    prefix_id: Optional[int] = None  # sequences with the same id share a cached prefix

    @property
    def kv_tokens(self) -> int:
        return self.prompt_len + self.output_len


def _split(group: List[SeqRequest], cap: Optional[int]) -> List[List[SeqRequest]]:
    """`group` cut into the fewest pieces of at most `cap` KV tokens (a
    sequence heavier than `cap` is a piece of its own), filled longest-first
    onto the lightest piece."""
    total = sum(r.kv_tokens for r in group)
    if cap is None or cap <= 0 or total <= cap:
        return [group]
    n = -(-total // cap)
    pieces: List[List[SeqRequest]] = [[] for _ in range(n)]
    load = [0] * n
    for r in sorted(group, key=lambda r: (-r.kv_tokens, r.seq_id)):
        k = min(range(n), key=lambda i: (load[i], i))
        pieces[k].append(r)
        load[k] += r.kv_tokens
    return [p for p in pieces if p]


def _groups(requests: Iterable[SeqRequest], cap: Optional[int] = None) -> List[List[SeqRequest]]:
    """Prefix groups (kept together up to `cap` KV tokens) and singletons,
    heaviest first; ties by smallest sequence id, so the order is
    deterministic."""
    by_prefix: Dict[int, List[SeqRequest]] = {}
    groups: List[List[SeqRequest]] = []
    for r in requests:
        if r.prefix_id is None:
            groups.append([r])
        else:
            by_prefix.setdefault(r.prefix_id, []).append(r)
    for pid in sorted(by_prefix):
        groups.extend(_split(by_prefix[pid], cap))
    for g in groups:
        g.sort(key=lambda r: r.seq_id)
    groups.sort(key=lambda g: (-sum(r.kv_tokens for r in g), g[0].seq_id))
    return groups


def _place(groups: List[List[SeqRequest]], ranks: Sequence[int], load: Dict[int, int],
           plan: Dict[int, List[int]], kv_budget: Optional[int]) -> None:
    for g in groups:
        need = sum(r.kv_tokens for r in g)
        target = min(ranks, key=lambda k: (load[k], k))
        if kv_budget is not None and load[target] + need > kv_budget:
            raise ValueError(f"sequences {[r.seq_id for r in g]} ({need} KV tokens) do not fit any rank's "
                             f"budget of {kv_budget} KV tokens")
        load[target] += need
        plan[target].extend(r.seq_id for r in g)


def plan_shards(requests: Sequence[SeqRequest], world: int,
                kv_budget: Optional[int] = None) -> List[List[int]]:
    """Sequence ids per rank (each list ascending). Raises ValueError when a
    sequence (or prefix group) fits no rank's remaining KV-token budget."""
    if world < 1:
        raise ValueError("world must be >= 1")
    ids = [r.seq_id for r in requests]
    if len(set(ids)) != len(ids):
        raise ValueError("duplicate sequence ids")
    plan: Dict[int, List[int]] = {k: [] for k in range(world)}
    load = {k: 0 for k in range(world)}
    fair = -(-sum(r.kv_tokens for r in requests) // world)
    _place(_groups(requests, fair), list(range(world)), load, plan, kv_budget)
    return [sorted(plan[k]) for k in range(world)]


def rank_load(plan: Sequence[Sequence[int]], requests: Sequence[SeqRequest]) -> List[int]:
    by_id = {r.seq_id: r for r in requests}
    return [sum(by_id[s].kv_tokens for s in shard) for shard in plan]


def requeue(plan: Sequence[Sequence[int]], requests: Sequence[SeqRequest], failed: Iterable[int],
            kv_budget: Optional[int] = None) -> List[List[int]]:
    """The plan with the failed ranks' sequences moved onto the survivors
    (longest-first onto the least-loaded survivor, prefix groups together);
    failed ranks end up empty. Raises ValueError when no rank survives."""
    failed = set(failed)
    world = len(plan)
    survivors = [k for k in range(world) if k not in failed]
    if not survivors:
        raise ValueError("no surviving rank to requeue onto")
    by_id = {r.seq_id: r for r in requests}
    new_plan = {k: (list(plan[k]) if k not in failed else []) for k in range(world)}
    load = {k: sum(by_id[s].kv_tokens for s in new_plan[k]) for k in range(world)}
    moved = [by_id[s] for k in sorted(failed) for s in plan[k]]
    fair = -(-(sum(load.values()) + sum(r.kv_tokens for r in moved)) // len(survivors))
    _place(_groups(moved, fair), survivors, load, new_plan, kv_budget)
    return [sorted(new_plan[k]) for k in range(world)]


def run_with_failover(store, rank: int, world: int, requests: Sequence[SeqRequest],
                      process: Callable[[int], object], deadline_s: float = 30.0,
                      poll_s: float = 0.05, kv_budget: Optional[int] = None
                      ) -> Tuple[Dict[int, object], List[int]]:
    """Serve this rank's shard of `plan_shards(requests, world)` with
    `process(seq_id)` (JSON-serialisable results) and return (results of all
    sequences, failed ranks). If this rank's own work raises, `fail/<rank>`
    is published and the exception propagates.

    Every rank measures the deadline from one common start: the wall-clock
    time of the first rank to enter (`t0`, written once with compare_set).
    Every rank agrees on one failed set: the first rank to decide (all ranks
    reported, or the deadline passed) writes `failed` with compare_set and
    every rank reads that value back, so survivors never requeue different
    sets. A rank that was slow but alive and finds itself in the agreed set
    discards its own results (the survivors serve its sequences again) and
    returns the survivors' merged results."""
    plan = plan_shards(requests, world, kv_budget)
    t0 = float(store.compare_set("t0", "", repr(time.time())).decode())
    deadline = t0 + deadline_s
    results: Dict[int, object] = {}
    try:
        for sid in plan[rank]:
            results[sid] = process(sid)
    except BaseException as exc:
        store.set(f"fail/{rank}", repr(exc))
        raise
    store.set(f"done/{rank}", json.dumps({str(k): v for k, v in results.items()}))

    agreed = None
    status: Dict[int, str] = {}
    while agreed is None:
        if store.check(["failed"]):
            agreed = store.get("failed").decode()
            break
        for r in range(world):
            if r in status:
                continue
            if store.check([f"done/{r}"]):
                status[r] = "done"
            elif store.check([f"fail/{r}"]):
                status[r] = "fail"
        if len(status) == world or time.time() > deadline:
            mine = sorted(r for r in range(world) if status.get(r) != "done")
            agreed = store.compare_set("failed", "", json.dumps(mine)).decode()
            break
        time.sleep(poll_s)
    failed = sorted(int(r) for r in json.loads(agreed))
    survivors = [r for r in range(world) if r not in failed]

    merged: Dict[int, object] = {}
    for r in survivors:
        merged.update({int(k): v for k, v in json.loads(store.get(f"done/{r}")).items()})
    if failed:
        plan2 = requeue(plan, requests, failed, kv_budget)
        if rank in survivors:
            extra = {sid: process(sid) for sid in plan2[rank] if sid not in plan[rank]}
            store.set(f"requeued/{rank}", json.dumps({str(k): v for k, v in extra.items()}))
        for r in survivors:
            key = f"requeued/{r}"
            while not store.check([key]):
                if time.time() > deadline + deadline_s:
                    raise TimeoutError(f"rank {r} did not publish its requeued results")
                time.sleep(poll_s)
            merged.update({int(k): v for k, v in json.loads(store.get(key)).items()})
    return merged, failed
