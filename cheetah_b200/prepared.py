"""Prepared-model directories: the format `cheetah init` writes and the
native backend reads.

Layout (written by the reference's `cheetah_init.c:1331-1452` and read by
`src/chat/native/store.rs:74-157`):

* ``<dir>/.cheetah/weights/layer_<N>.safetensors`` for every tensor whose
  name carries ``layers.<N>.`` and ``global.safetensors`` for the rest
  (``cheetah_init.c:859-871``);
* every payload starts on a 4096-byte boundary inside the data section
  (gaps are named ``__cheetah_padding_<n>`` U8 tensors), and the header is
  space-padded so the data section itself starts on a 4096-byte boundary;
* ``<dir>/cheetah_units.json``: one record per tensor with ``unit_id``,
  ``dtype``, ``shape``, ``bytes``, ``source_file``, ``source_offset``
  (relative to the shard's data section), ``layer_id``
  (``cheetah_init.c:1668-1716``);
* ``<dir>/config.json`` copied from the source checkpoint.

This module also generates the seeded synthetic Qwen2 checkpoints the
benchmarks and parity tests run on (random-init bf16 N(0, 0.02) from seed 0,
one child seed per tensor chunk), either directly in the prepared layout or
in the Hugging Face single-file layout that `cheetah init` converts.
"""

from __future__ import annotations

import dataclasses
import json
import os
import struct
from pathlib import Path
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np

ALIGNMENT = 4096
UNITS_FILENAME = "cheetah_units.json"  # src/ant.rs:39

DTYPE_BYTES = {"BF16": 2, "F16": 2, "F32": 4, "U8": 1, "I8": 1}


@dataclasses.dataclass(frozen=True)
class Qwen2Shape:
    """Qwen2-family decoder hyper-parameters (`qwen2.rs:66-82` profiles)."""

    hidden_size: int
    num_layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    tie_word_embeddings: bool = True
    max_position_embeddings: int = 32768
    attention_bias: bool = True

    @property
    def q_dim(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def config_json(self) -> dict:
        return {
            "architectures": ["Qwen2ForCausalLM"],
            "model_type": "qwen2",
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.q_heads,
            "num_key_value_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "vocab_size": self.vocab_size,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_eps,
            "tie_word_embeddings": self.tie_word_embeddings,
            "use_sliding_window": False,
            "sliding_window": 32768,
            "max_position_embeddings": self.max_position_embeddings,
            "hidden_act": "silu",
            "torch_dtype": "bfloat16",
        }


# Qwen2-0.5B and Qwen2-7B architectures (qwen2.rs:72-74 profiles).
QWEN2_0_5B = Qwen2Shape(896, 24, 14, 2, 64, 4864, 151936)
QWEN2_7B = Qwen2Shape(3584, 28, 28, 4, 128, 18944, 152064, tie_word_embeddings=False)
# Small shapes with the real head geometry (7:1 GQA, head_dim 64 / 128) for
# parity tests the CPU oracle finishes in seconds.
TINY = Qwen2Shape(256, 2, 14, 2, 64, 512, 1000, max_position_embeddings=4096)
TINY_7B_HEADS = Qwen2Shape(512, 2, 28, 4, 128, 768, 1024, tie_word_embeddings=False,
                           max_position_embeddings=4096)
TINY_WIDE_MLP = Qwen2Shape(256, 2, 14, 2, 64, 16384, 1000, max_position_embeddings=4096)
TINY_15B_HEADS = Qwen2Shape(1536, 2, 12, 2, 128, 2048, 1024, tie_word_embeddings=False,
                            max_position_embeddings=4096)


def tensor_specs(shape: Qwen2Shape) -> List[Tuple[str, Tuple[int, ...]]]:
    """Every HF-layout tensor of a Qwen2 checkpoint, sorted by name."""
    specs: List[Tuple[str, Tuple[int, ...]]] = [
        ("model.embed_tokens.weight", (shape.vocab_size, shape.hidden_size)),
        ("model.norm.weight", (shape.hidden_size,)),
    ]
    if not shape.tie_word_embeddings:
        specs.append(("lm_head.weight", (shape.vocab_size, shape.hidden_size)))
    h, q, kv, inter = shape.hidden_size, shape.q_dim, shape.kv_dim, shape.intermediate_size
    for layer in range(shape.num_layers):
        p = f"model.layers.{layer}."
        specs += [
            (p + "input_layernorm.weight", (h,)),
            (p + "post_attention_layernorm.weight", (h,)),
            (p + "self_attn.q_proj.weight", (q, h)),
            (p + "self_attn.k_proj.weight", (kv, h)),
            (p + "self_attn.v_proj.weight", (kv, h)),
            (p + "self_attn.o_proj.weight", (h, q)),
            (p + "mlp.gate_proj.weight", (inter, h)),
            (p + "mlp.up_proj.weight", (inter, h)),
            (p + "mlp.down_proj.weight", (h, inter)),
        ]
        if shape.attention_bias:
            specs += [
                (p + "self_attn.q_proj.bias", (q,)),
                (p + "self_attn.k_proj.bias", (kv,)),
                (p + "self_attn.v_proj.bias", (kv,)),
            ]
    specs.sort(key=lambda item: item[0])
    return specs


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounding = ((bits >> 16) & 1) + np.uint32(0x7FFF)
    return ((bits + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact bf16 -> f32 widening (`ops.rs:59-62`)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def generate_tensors(shape: Qwen2Shape, seed: int = 0, std: float = 0.02,
                     chunk: int = 1 << 24, threads: Optional[int] = None
                     ) -> Iterator[Tuple[str, Tuple[int, ...], np.ndarray]]:
    """Seeded random-init weights: N(0, std) bf16 for every tensor (norms and
    biases included), yielded in sorted-name order. Tensor i's chunk j of
    `chunk` values is drawn from its own generator, seeded by child (i, j) of
    `SeedSequence(seed)`, so the values do not depend on how many threads
    draw them; the chunks are drawn on a thread pool (numpy releases the GIL
    while it fills large arrays)."""
    from concurrent.futures import ThreadPoolExecutor

    specs = tensor_specs(shape)
    root = np.random.SeedSequence(seed)
    per_tensor = root.spawn(len(specs))
    outs = [np.empty(int(np.prod(dims)), dtype=np.uint16) for _, dims in specs]
    jobs = []
    for i, (_, dims) in enumerate(specs):
        count = outs[i].size
        seeds = per_tensor[i].spawn(max(1, -(-count // chunk)))
        for j, start in enumerate(range(0, count, chunk)):
            jobs.append((i, start, min(chunk, count - start), seeds[j]))

    def draw(job):
        i, start, n, ss = job
        values = np.random.default_rng(ss).standard_normal(n, dtype=np.float32)
        values *= np.float32(std)
        outs[i][start:start + n] = f32_to_bf16_bits(values)

    with ThreadPoolExecutor(max_workers=threads or min(32, os.cpu_count() or 1)) as pool:
        list(pool.map(draw, jobs))
    for (name, dims), out in zip(specs, outs):
        yield name, dims, out


def _shard_name(tensor_name: str) -> str:
    """`cheetah_init.c:859-871`: layer_<N>.safetensors or global.safetensors."""
    marker = tensor_name.find("layers.")
    if marker >= 0:
        digits = ""
        for ch in tensor_name[marker + len("layers."):]:
            if ch.isdigit():
                digits += ch
            else:
                break
        if digits:
            return f"layer_{int(digits)}.safetensors"
    return "global.safetensors"


def _layer_id(tensor_name: str) -> int:
    marker = tensor_name.find("layers.")
    if marker < 0:
        return 0
    digits = ""
    for ch in tensor_name[marker + len("layers."):]:
        if ch.isdigit():
            digits += ch
        else:
            break
    return int(digits) if digits else 0


def write_safetensors(path: Path, tensors: Sequence[Tuple[str, str, Tuple[int, ...], np.ndarray]],
                      aligned: bool) -> Dict[str, int]:
    """Write a safetensors file. With ``aligned`` every payload offset and the
    data section start are 4096-byte aligned the way `cheetah init` pads them.
    Returns each tensor's offset relative to the data section."""
    header: Dict[str, dict] = {}
    offsets: Dict[str, int] = {}
    cursor = 0
    pad_index = 0
    layout: List[Tuple[int, Optional[np.ndarray]]] = []
    for name, dtype, dims, data in tensors:
        nbytes = int(np.asarray(data).nbytes)
        if aligned:
            padding = (ALIGNMENT - cursor % ALIGNMENT) % ALIGNMENT
            if padding:
                header[f"__cheetah_padding_{pad_index:06d}"] = {
                    "dtype": "U8", "shape": [padding], "data_offsets": [cursor, cursor + padding]}
                pad_index += 1
                layout.append((padding, None))
                cursor += padding
        header[name] = {"dtype": dtype, "shape": list(dims), "data_offsets": [cursor, cursor + nbytes]}
        offsets[name] = cursor
        layout.append((nbytes, data))
        cursor += nbytes
    text = json.dumps(header, separators=(",", ":")).encode()
    if aligned:
        data_start = (len(text) + 8 + ALIGNMENT - 1) & ~(ALIGNMENT - 1)
        text = text + b" " * (data_start - 8 - len(text))
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for nbytes, data in layout:
            if data is None:
                f.write(b"\0" * nbytes)
            else:
                f.write(np.ascontiguousarray(data).tobytes())
    return offsets


def write_prepared(dst: os.PathLike, shape: Qwen2Shape, seed: int = 0,
                   tensors: Optional[Iterator[Tuple[str, Tuple[int, ...], np.ndarray]]] = None) -> Path:
    """Write a seeded synthetic Qwen2 model directly in the prepared layout."""
    dst = Path(dst)
    weights = dst / ".cheetah" / "weights"
    weights.mkdir(parents=True, exist_ok=True)
    source = tensors if tensors is not None else generate_tensors(shape, seed)
    by_shard: Dict[str, List[Tuple[str, str, Tuple[int, ...], np.ndarray]]] = {}
    order: List[Tuple[str, str, Tuple[int, ...], int]] = []
    for name, dims, data in source:
        shard = _shard_name(name)
        by_shard.setdefault(shard, []).append((name, "BF16", dims, data))
        order.append((name, shard, dims, int(data.nbytes)))
    offsets: Dict[str, int] = {}
    for shard, items in by_shard.items():
        offsets.update(write_safetensors(weights / shard, items, aligned=True))
        by_shard[shard] = []  # release payload references early
    units = [
        {
            "unit_id": name, "name": name, "dtype": "BF16", "shape": list(dims),
            "bytes": nbytes, "source_file": shard, "source_offset": offsets[name],
            "shard": shard, "layer_id": _layer_id(name),
        }
        for name, shard, dims, nbytes in order
    ]
    (dst / UNITS_FILENAME).write_text(json.dumps(units, indent=1))
    (dst / "config.json").write_text(json.dumps(shape.config_json(), indent=1))
    return dst


def write_hf_source(dst: os.PathLike, shape: Qwen2Shape, seed: int = 0) -> Path:
    """Seeded synthetic checkpoint in the Hugging Face layout (one
    model.safetensors + config.json + a minimal tokenizer.json), the input
    `cheetah init` converts into the prepared layout."""
    dst = Path(dst)
    dst.mkdir(parents=True, exist_ok=True)
    items = [(name, "BF16", dims, data) for name, dims, data in generate_tensors(shape, seed)]
    write_safetensors(dst / "model.safetensors", items, aligned=False)
    (dst / "config.json").write_text(json.dumps(shape.config_json(), indent=1))
    tokenizer = {"version": "1.0", "model": {"type": "WordLevel", "vocab": {"<|endoftext|>": 0},
                                             "unk_token": "<|endoftext|>"},
                 "added_tokens": [{"id": 0, "content": "<|endoftext|>", "special": True}]}
    (dst / "tokenizer.json").write_text(json.dumps(tokenizer))
    return dst


@dataclasses.dataclass
class Unit:
    unit_id: str
    dtype: str
    shape: Tuple[int, ...]
    nbytes: int
    source_file: str
    source_offset: int
    layer_id: int
    data: np.ndarray  # raw bytes (uint8 memmap view)

    def array(self) -> np.ndarray:
        """Typed view: uint16 bit patterns for BF16/F16, float32 for F32."""
        if self.dtype in ("BF16", "F16"):
            return self.data.view(np.uint16).reshape(self.shape)
        if self.dtype == "F32":
            return self.data.view(np.float32).reshape(self.shape)
        return self.data

    def f32(self) -> np.ndarray:
        if self.dtype == "BF16":
            return bf16_bits_to_f32(self.array())
        if self.dtype == "F16":
            return self.array().view(np.float16).astype(np.float32)
        return np.array(self.array(), dtype=np.float32)


class PreparedModel:
    """Read side of the prepared layout (`store.rs:74-157`): the units
    manifest resolves each unit to a byte range inside a memory-mapped shard
    (offset = 8 + header length + source_offset)."""

    def __init__(self, root: os.PathLike):
        self.root = Path(root)
        manifest = self.root / UNITS_FILENAME
        records = json.loads(manifest.read_text())
        if not records:
            raise ValueError("Ant units manifest is empty; run `cheetah init` first.")
        weights = self.root / ".cheetah" / "weights"
        maps: Dict[str, Tuple[np.memmap, int]] = {}
        self.units: Dict[str, Unit] = {}
        for rec in records:
            if not rec.get("unit_id") or not rec.get("source_file"):
                continue
            shard = rec["source_file"]
            if shard not in maps:
                mm = np.memmap(weights / shard, dtype=np.uint8, mode="r")
                if mm.shape[0] < 8:
                    raise ValueError(f"Shard {shard} is too small for a header.")
                header_len = int.from_bytes(bytes(mm[:8]), "little")
                data_start = 8 + header_len
                if data_start > mm.shape[0]:
                    raise ValueError(f"Shard {shard} header exceeds the file size.")
                maps[shard] = (mm, data_start)
            mm, data_start = maps[shard]
            start = data_start + int(rec["source_offset"])
            end = start + int(rec.get("bytes", 0))
            if int(rec["source_offset"]) + int(rec.get("bytes", 0)) > mm.shape[0]:
                raise ValueError(f"Unit {rec['unit_id']} exceeds the bounds of shard {shard}.")
            self.units[rec["unit_id"]] = Unit(
                rec["unit_id"], rec.get("dtype", ""), tuple(rec.get("shape", [])),
                int(rec.get("bytes", 0)), shard, int(rec["source_offset"]),
                int(rec.get("layer_id", 0)), mm[start:end])
        config_path = self.root / "config.json"
        self.raw_config = json.loads(config_path.read_text()) if config_path.exists() else {}

    def __contains__(self, unit_id: str) -> bool:
        return unit_id in self.units

    def unit(self, unit_id: str) -> Unit:
        try:
            return self.units[unit_id]
        except KeyError:
            raise KeyError(f"Native backend: unknown unit '{unit_id}'.") from None

    def max_layer_id(self) -> int:
        return max((u.layer_id for u in self.units.values()), default=0)


# Qwen2 family constants (qwen2.rs:66-82).
QWEN2_FAMILY = {
    "rope_theta": 1_000_000.0,
    "rms_norm_eps": 1e-6,
    "tie_word_embeddings": True,
    "profiles": [(896, 151936, 14, 2, 64), (1536, 151936, 12, 2, 128), (3584, 152064, 28, 4, 128)],
}


def resolve_config(model: PreparedModel, max_positions: Optional[int] = None) -> dict:
    """Qwen2 subset of `DecoderConfig::resolve` (`decoder.rs:260-486`):
    config.json first, then the units manifest's shapes, then the family
    constants. Returns the fields of `CheetahCudaConfig`."""
    raw = model.raw_config
    embed = model.units.get("model.embed_tokens.weight")
    hidden = raw.get("hidden_size") or (embed.shape[1] if embed else None)
    vocab = raw.get("vocab_size") or (embed.shape[0] if embed else None)
    layers = raw.get("num_hidden_layers") or (model.max_layer_id() + 1)
    profile = next((p for p in QWEN2_FAMILY["profiles"] if p[0] == hidden), None)
    q_heads = raw.get("num_attention_heads") or (profile[2] if profile else None)
    kv_heads = raw.get("num_key_value_heads") or (profile[3] if profile else q_heads)
    head_dim = raw.get("head_dim") or (hidden // q_heads if hidden and q_heads else None)
    gate = model.units.get("model.layers.0.mlp.gate_proj.weight")
    inter = raw.get("intermediate_size") or (gate.shape[0] if gate else None)
    if None in (hidden, vocab, q_heads, kv_heads, head_dim, inter):
        raise ValueError("Native backend: could not resolve the decoder configuration.")
    tie = raw.get("tie_word_embeddings", QWEN2_FAMILY["tie_word_embeddings"])
    if "lm_head.weight" in model.units and "tie_word_embeddings" not in raw:
        tie = False
    window = 0
    if raw.get("use_sliding_window", False) and raw.get("sliding_window"):
        window = int(raw["sliding_window"])
    max_pos = max_positions or int(raw.get("max_position_embeddings", 32768))
    return {
        "hidden_size": int(hidden), "num_layers": int(layers), "q_heads": int(q_heads),
        "kv_heads": int(kv_heads), "head_dim": int(head_dim), "rotary_dim": int(head_dim),
        "intermediate_size": int(inter), "vocab_size": int(vocab),
        "rms_eps": float(raw.get("rms_norm_eps", QWEN2_FAMILY["rms_norm_eps"])),
        "rope_theta": float(raw.get("rope_theta", QWEN2_FAMILY["rope_theta"])),
        "tie_word_embeddings": 1 if tie else 0, "sliding_window": window,
        "max_positions": int(max_pos),
    }


SHAPES = {"qwen2-0.5b": QWEN2_0_5B, "qwen2-7b": QWEN2_7B, "tiny": TINY, "tiny-7b-heads": TINY_7B_HEADS}


def cached_synthetic_path(name: str, seed: int = 0, root: Optional[os.PathLike] = None) -> Path:
    """Where `cached_synthetic` keeps the model (complete once `.complete` exists)."""
    base = Path(root or os.environ.get("CHEETAH_MODEL_CACHE", "/tmp/cheetah_models"))
    return base / f"{name}_seed{seed}"


def cached_synthetic(name: str, seed: int = 0, root: Optional[os.PathLike] = None) -> Path:
    """Seeded synthetic prepared model, written once per machine under
    `$CHEETAH_MODEL_CACHE` (default /tmp/cheetah_models) and reused."""
    target = cached_synthetic_path(name, seed, root)
    base = target.parent
    marker = target / ".complete"
    if marker.exists():
        return target
    tmp = base / f".{name}_seed{seed}.{os.getpid()}"
    if tmp.exists():
        import shutil
        shutil.rmtree(tmp)
    write_prepared(tmp, SHAPES[name], seed)
    (tmp / ".complete").write_text("ok")
    try:
        os.rename(tmp, target)
    except OSError:
        import shutil
        shutil.rmtree(tmp, ignore_errors=True)
    return target
