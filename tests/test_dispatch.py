"""Sequence dispatch over ranks: placement by KV-token load, prefix-group
co-location, requeue after a rank failure, and the store-based failover run
as world-size-2 CPU processes (gloo process group, TCPStore on 127.0.0.1).
Failures are made on the host: a rank whose work raises, a rank that exits
without reporting, and a rank that is alive but finishes after the deadline.
No GPU is involved."""

from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest

from cheetah_b200.dispatch import SeqRequest, plan_shards, rank_load, requeue, run_with_failover


def serve_requests(n_seq: int = 64):
    """The serving workload's sequences (seed 2: prompts U[128, 8192],
    outputs U[32, 512], half share a 1024-token prefix)."""
    rng = np.random.default_rng(2)
    prompt_len = rng.integers(128, 8193, n_seq)
    out_len = rng.integers(32, 513, n_seq)
    shared = set(rng.permutation(n_seq)[: n_seq // 2].tolist())
    return [SeqRequest(i, int(prompt_len[i]), int(out_len[i]),
                       0 if (i in shared and prompt_len[i] > 1024) else None) for i in range(n_seq)]


def check_partition(plan, requests):
    placed = sorted(s for shard in plan for s in shard)
    assert placed == sorted(r.seq_id for r in requests)
    for shard in plan:
        assert shard == sorted(shard)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_is_a_balanced_partition(world):
    reqs = serve_requests()
    plan = plan_shards(reqs, world)
    check_partition(plan, reqs)
    load = rank_load(plan, reqs)
    heaviest = max(r.kv_tokens for r in reqs)
    # Greedy onto the lightest rank: no rank exceeds the mean by more than
    # one placed unit, and a prefix piece is at most the mean itself.
    mean = sum(load) / world
    assert max(load) <= mean + max(heaviest, mean)
    assert max(load) - min(load) <= max(heaviest, -(-sum(load) // world))
    assert plan == plan_shards(list(reversed(reqs)), world)  # order-independent


def test_prefix_group_stays_together_when_it_fits():
    reqs = [SeqRequest(i, 100 * (i + 1), 10, 7 if i in (1, 4, 6) else None) for i in range(8)]
    plan = plan_shards(reqs, 2)
    check_partition(plan, reqs)
    holders = [k for k, shard in enumerate(plan) if {1, 4, 6} & set(shard)]
    assert len(holders) == 1 and {1, 4, 6} <= set(plan[holders[0]])


def test_heavy_prefix_group_is_split_into_fewest_pieces():
    # One group of 8 equal sequences, 4 ranks: pieces of at most the mean
    # load, so each rank carries two of them and pays one prefix prefill.
    reqs = [SeqRequest(i, 1000, 0, 3) for i in range(8)]
    plan = plan_shards(reqs, 4)
    check_partition(plan, reqs)
    assert [len(s) for s in plan] == [2, 2, 2, 2]
    reqs8 = serve_requests()
    plan8 = plan_shards(reqs8, 8)
    grouped = {r.seq_id for r in reqs8 if r.prefix_id is not None}
    holders = [k for k, shard in enumerate(plan8) if grouped & set(shard)]
    fair = -(-sum(r.kv_tokens for r in reqs8) // 8)
    group_load = sum(r.kv_tokens for r in reqs8 if r.seq_id in grouped)
    assert 1 < len(holders) <= -(-group_load // fair)
    assert max(rank_load(plan8, reqs8)) <= 1.05 * fair


def test_longest_first_onto_lightest_rank():
    reqs = [SeqRequest(0, 10, 0), SeqRequest(1, 50, 0), SeqRequest(2, 40, 0), SeqRequest(3, 30, 0)]
    # 50 -> r0, 40 -> r1, 30 -> r1 (40 < 50), 10 -> r0 (50 < 70)
    assert plan_shards(reqs, 2) == [[0, 1], [2, 3]]


def test_kv_budget_is_enforced():
    reqs = [SeqRequest(i, 1000, 100) for i in range(4)]
    assert rank_load(plan_shards(reqs, 2, kv_budget=2200), reqs) == [2200, 2200]
    with pytest.raises(ValueError, match="budget"):
        plan_shards(reqs, 2, kv_budget=2199)
    with pytest.raises(ValueError, match="duplicate"):
        plan_shards(reqs + [SeqRequest(0, 1, 1)], 2)
    with pytest.raises(ValueError):
        plan_shards(reqs, 0)


@pytest.mark.parametrize("world,failed", [(2, [1]), (2, [0]), (4, [2]), (8, [0, 5, 7])])
def test_requeue_moves_only_the_failed_ranks_sequences(world, failed):
    reqs = serve_requests()
    plan = plan_shards(reqs, world)
    plan2 = requeue(plan, reqs, failed)
    check_partition(plan2, reqs)
    for k in range(world):
        if k in failed:
            assert plan2[k] == []
        else:
            assert set(plan[k]) <= set(plan2[k])
    survivors = world - len(failed)
    load = [x for k, x in enumerate(rank_load(plan2, reqs)) if k not in failed]
    assert max(load) - min(load) <= 2 * sum(load) / survivors
    with pytest.raises(ValueError, match="surviving"):
        requeue(plan, reqs, range(world))


# ---------------------------------------------------------------------------
# world-size-2 runs as spawned processes

N_SEQ = 12


def small_requests():
    return [SeqRequest(i, 64 + 37 * i % 200, 8 + i % 5, 1 if i % 3 == 0 else None) for i in range(N_SEQ)]


def work(sid: int) -> int:
    return sid * sid + 1


def _rank_main(rank: int, world: int, port: int, mode: str, deadline_s: float) -> None:
    import torch
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world + 1, is_master=False, timeout=timedelta(seconds=20))
    if mode == "ok":
        dist.init_process_group("gloo", store=dist.PrefixStore("pg", store), rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
    if mode == "exit" and rank == 1:
        os._exit(3)  # never reports: the survivors find out by the deadline
    calls = []

    def process(sid):
        calls.append(sid)
        if mode == "raise" and rank == 1 and len(calls) == 2:
            raise RuntimeError("injected failure on the host")
        if mode == "slow" and rank == world - 1 and len(calls) == 1:
            time.sleep(deadline_s + 2.0)  # alive, but past every other rank's deadline
        return work(sid)

    merged, failed = run_with_failover(store, rank, world, small_requests(), process,
                                       deadline_s=deadline_s, poll_s=0.02)
    if mode == "ok":
        # the bench's reduction of per-rank counts over the process group
        t = torch.tensor([float(len(calls))])
        dist.all_reduce(t)
        store.set(f"total/{rank}", str(int(t.item())))
        dist.destroy_process_group()
    store.set(f"result/{rank}", json.dumps({"merged": {str(k): v for k, v in merged.items()},
                                            "failed": failed, "calls": calls}))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_world(mode: str, world: int = 2, deadline_s: float = 20.0):
    import torch.distributed as dist
    port = _free_port()
    store = dist.TCPStore("127.0.0.1", port, world + 1, is_master=True, timeout=timedelta(seconds=60),
                          wait_for_workers=False)
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, deadline_s)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    codes = [p.exitcode for p in procs]
    out = {}
    for r in range(world):
        if store.check([f"result/{r}"]):
            out[r] = json.loads(store.get(f"result/{r}"))
    return store, codes, out


def run_world2(mode: str, deadline_s: float = 20.0):
    return run_world(mode, 2, deadline_s)


def test_world2_all_ranks_succeed():
    store, codes, out = run_world2("ok")
    assert codes == [0, 0]
    plan = plan_shards(small_requests(), 2)
    expect = {str(i): work(i) for i in range(N_SEQ)}
    for r in range(2):
        assert out[r]["failed"] == []
        assert out[r]["merged"] == expect
        assert out[r]["calls"] == plan[r]
        assert int(store.get(f"total/{r}")) == N_SEQ


def test_world2_rank_that_raises_is_requeued():
    store, codes, out = run_world2("raise")
    assert codes[0] == 0 and codes[1] != 0
    assert 1 not in out
    assert store.check(["fail/1"]) and not store.check(["done/1"])
    assert "injected failure" in store.get("fail/1").decode()
    plan = plan_shards(small_requests(), 2)
    assert out[0]["failed"] == [1]
    assert out[0]["merged"] == {str(i): work(i) for i in range(N_SEQ)}
    # rank 0 served its own shard first, then every sequence of rank 1
    assert out[0]["calls"] == plan[0] + plan[1]


def test_world2_rank_that_never_reports_times_out_and_is_requeued():
    store, codes, out = run_world2("exit", deadline_s=3.0)
    assert codes == [0, 3]
    assert not store.check(["fail/1"]) and not store.check(["done/1"])
    assert out[0]["failed"] == [1]
    assert out[0]["merged"] == {str(i): work(i) for i in range(N_SEQ)}


def test_requeue_respects_the_kv_budget():
    reqs = [SeqRequest(i, 900, 100) for i in range(6)]   # 1000 KV tokens each
    plan = plan_shards(reqs, 3, kv_budget=2000)           # two per rank
    assert rank_load(plan, reqs) == [2000, 2000, 2000]
    with pytest.raises(ValueError, match="budget"):
        requeue(plan, reqs, [1], kv_budget=2000)         # survivors are full
    plan2 = requeue(plan, reqs, [1], kv_budget=3000)
    check_partition(plan2, reqs)
    assert rank_load(plan2, reqs) == [3000, 0, 3000]


@pytest.mark.parametrize("world", [2, 3])
def test_slow_rank_past_the_deadline_every_rank_agrees(world):
    """The last rank sleeps past the common deadline and still finishes: every
    rank (the slow one included) uses the one agreed failed set, the slow
    rank's sequences are served again by the survivors, and nobody times
    out waiting for a requeue that was never published."""
    store, codes, out = run_world("slow", world, deadline_s=3.0)
    assert codes == [0] * world
    slow = world - 1
    expect = {str(i): work(i) for i in range(N_SEQ)}
    assert json.loads(store.get("failed")) == [slow]
    plan = plan_shards(small_requests(), world)
    plan2 = requeue(plan, small_requests(), [slow])
    for r in range(world):
        assert out[r]["failed"] == [slow]
        assert out[r]["merged"] == expect
    for r in range(slow):
        assert out[r]["calls"] == plan[r] + [s for s in plan2[r] if s not in plan[r]]
    assert out[slow]["calls"] == plan[slow]
