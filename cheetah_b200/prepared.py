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
class DecoderShape:
    """Hyper-parameters of a dense llama-shaped decoder: Qwen2 (`qwen2.rs:66-82`
    profiles) and the families that differ from it only by composition:
    llama (no attention biases, `llama.rs:66-82`), mistral (a decode-time
    sliding window, `mistral.rs:63-77`) and qwen3 (per-head q/k RMSNorm units,
    `qwen3.rs:62-77`)."""

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
    family: str = "qwen2"
    sliding_window: int = 0     # written to config.json for the non-qwen2 families
    qk_norm: bool = False       # qwen3: self_attn.{q,k}_norm.weight [head_dim] units

    @property
    def q_dim(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def config_json(self) -> dict:
        cfg = {
            "architectures": [FAMILIES[self.family]["architectures"][0]],
            "model_type": self.family,
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
            "max_position_embeddings": self.max_position_embeddings,
            "hidden_act": "silu",
            "torch_dtype": "bfloat16",
        }
        if self.family == "qwen2":
            # Qwen2 configs carry a window the modeling never engages.
            cfg.update(use_sliding_window=False, sliding_window=32768)
        elif self.sliding_window:
            cfg["sliding_window"] = self.sliding_window  # `use_sliding_window` absent = on
        return cfg


Qwen2Shape = DecoderShape


# Qwen2-0.5B and Qwen2-7B architectures (qwen2.rs:72-74 profiles).
QWEN2_0_5B = DecoderShape(896, 24, 14, 2, 64, 4864, 151936)
QWEN2_7B = DecoderShape(3584, 28, 28, 4, 128, 18944, 152064, tie_word_embeddings=False)
# Small shapes with the real head geometry (7:1 GQA, head_dim 64 / 128) for
# parity tests the CPU oracle finishes in seconds.
TINY = DecoderShape(256, 2, 14, 2, 64, 512, 1000, max_position_embeddings=4096)
TINY_7B_HEADS = DecoderShape(512, 2, 28, 4, 128, 768, 1024, tie_word_embeddings=False,
                             max_position_embeddings=4096)
TINY_WIDE_MLP = DecoderShape(256, 2, 14, 2, 64, 16384, 1000, max_position_embeddings=4096)
TINY_15B_HEADS = DecoderShape(1536, 2, 12, 2, 128, 2048, 1024, tie_word_embeddings=False,
                              max_position_embeddings=4096)
# The other dense families at small sizes: llama (multi-head, no biases, rope
# theta 1e4, eps 1e-5, untied), mistral (4:1 GQA, a 48-token window so short
# prompts engage it), qwen3 (head_dim 128 > hidden / heads, q/k norms, tied).
TINY_LLAMA = DecoderShape(256, 2, 4, 4, 64, 512, 1000, rope_theta=10_000.0, rms_eps=1e-5,
                          tie_word_embeddings=False, max_position_embeddings=4096,
                          attention_bias=False, family="llama")
TINY_MISTRAL = DecoderShape(256, 2, 8, 2, 64, 512, 1000, rope_theta=10_000.0, rms_eps=1e-5,
                            tie_word_embeddings=False, max_position_embeddings=4096,
                            attention_bias=False, family="mistral", sliding_window=48)
TINY_QWEN3 = DecoderShape(256, 2, 8, 4, 128, 512, 1000, max_position_embeddings=4096,
                          attention_bias=False, family="qwen3", qk_norm=True)
# Llama-3.2-1B's architecture (`llama.rs:72` profile; tied head as published).
LLAMA_1B = DecoderShape(2048, 16, 32, 8, 64, 8192, 128256, rope_theta=500_000.0, rms_eps=1e-5,
                        tie_word_embeddings=True, max_position_embeddings=4096,
                        attention_bias=False, family="llama")


def tensor_specs(shape: DecoderShape) -> List[Tuple[str, Tuple[int, ...]]]:
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
        if shape.qk_norm:
            specs += [
                (p + "self_attn.q_norm.weight", (shape.head_dim,)),
                (p + "self_attn.k_norm.weight", (shape.head_dim,)),
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


# qwen3's per-head q/k norm weights are drawn N(0, 1): with N(0, 0.02) the
# normalised q and k would be ~0.02 per element and every attention softmax
# near-uniform, so the norms (and RoPE after them) would barely reach the
# logits a parity test compares.
QK_NORM_SUFFIXES = ("self_attn.q_norm.weight", "self_attn.k_norm.weight")
QK_NORM_STD = 1.0


def generate_tensors(shape: DecoderShape, seed: int = 0, std: float = 0.02,
                     chunk: int = 1 << 24, threads: Optional[int] = None
                     ) -> Iterator[Tuple[str, Tuple[int, ...], np.ndarray]]:
    """Seeded random-init weights: N(0, std) bf16 for every tensor (norms and
    biases included; q/k norms N(0, QK_NORM_STD)), yielded in sorted-name order. Tensor i's chunk j of
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
        values *= np.float32(std if not specs[i][0].endswith(QK_NORM_SUFFIXES) else QK_NORM_STD)
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


def write_prepared(dst: os.PathLike, shape: DecoderShape, seed: int = 0,
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


def write_hf_source(dst: os.PathLike, shape: DecoderShape, seed: int = 0) -> Path:
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


# Family constants of the dense registrations this backend serves
# (`registrations/qwen2.rs:63-82`, `qwen3.rs:62-77`, `llama.rs:66-82`,
# `mistral.rs:63-77`): the architecture names that select them
# (`registry.rs:328`), rope theta, RMSNorm epsilon, tied head,
# (hidden, vocab, q heads, kv heads, head_dim) profiles, context cap.
FAMILIES = {
    "qwen2": {
        "architectures": ("Qwen2ForCausalLM", "qwen2"),
        "rope_theta": 1_000_000.0, "rms_norm_eps": 1e-6, "tie_word_embeddings": True,
        "profiles": [(896, 151936, 14, 2, 64), (1536, 151936, 12, 2, 128), (3584, 152064, 28, 4, 128)],
        "max_position_embeddings": None,
    },
    "qwen3": {
        "architectures": ("Qwen3ForCausalLM", "qwen3"),
        "rope_theta": 1_000_000.0, "rms_norm_eps": 1e-6, "tie_word_embeddings": True,
        "profiles": [(8192, 32768, 64, 8, 128)],
        "max_position_embeddings": None,
    },
    "llama": {
        "architectures": ("LlamaForCausalLM", "llama"),
        "rope_theta": 10_000.0, "rms_norm_eps": 1e-5, "tie_word_embeddings": False,
        "profiles": [(2048, 128256, 32, 8, 64), (3072, 128256, 24, 8, 128),
                     (4096, 128256, 32, 8, 128), (4096, 32000, 32, 32, 128)],
        "max_position_embeddings": 4096,
    },
    "mistral": {
        "architectures": ("MistralForCausalLM", "mistral"),
        "rope_theta": 10_000.0, "rms_norm_eps": 1e-5, "tie_word_embeddings": False,
        "profiles": [(4096, 32000, 32, 8, 128), (4096, 32768, 32, 8, 128)],
        "max_position_embeddings": 32768,
    },
}
QWEN2_FAMILY = FAMILIES["qwen2"]
# A config that names no architecture resolves against llama-shaped defaults
# (`decoder.rs:283-296`).
DEFAULT_FAMILY = {
    "architectures": (), "rope_theta": 1_000_000.0, "rms_norm_eps": 1e-6,
    "tie_word_embeddings": False, "profiles": [], "max_position_embeddings": None,
}


def config_architecture(raw: dict) -> Optional[str]:
    """First `architectures` entry, else `model_type` (`chat/mod.rs:62-67`)."""
    archs = raw.get("architectures")
    if isinstance(archs, list) and archs and isinstance(archs[0], str):
        return archs[0]
    mt = raw.get("model_type")
    return mt if isinstance(mt, str) else None


def family_for(raw: dict) -> Tuple[Optional[str], dict]:
    """(family name, constants) for a config.json; raises for an
    architecture outside the dense families this backend serves (gemma's
    offset norms, phi's fused QKV / LayerNorm / parallel residual, mixtral's
    experts are other compositions)."""
    arch = config_architecture(raw)
    if arch is None:
        return None, DEFAULT_FAMILY
    for name, fam in FAMILIES.items():
        if arch in fam["architectures"]:
            return name, fam
    raise ValueError(f"CUDA backend: architecture '{arch}' is not served "
                     f"(dense families: {', '.join(sorted(FAMILIES))}).")


def _field_u(raw: dict, name: str) -> Optional[int]:
    """`Value::as_u64`: a non-negative JSON integer, else None."""
    v = raw.get(name)
    return v if isinstance(v, int) and not isinstance(v, bool) and v >= 0 else None


def _field_f(raw: dict, name: str) -> Optional[float]:
    """`Value::as_f64`: any JSON number, else None."""
    v = raw.get(name)
    return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else None


def _field_b(raw: dict, name: str) -> Optional[bool]:
    v = raw.get(name)
    return v if isinstance(v, bool) else None


def resolve_config(model: PreparedModel, max_positions: Optional[int] = None) -> dict:
    """The dense subset of `DecoderConfig::resolve` (`decoder.rs:260-486`):
    config.json first, then the units manifest's shapes, then the family
    constants. Returns the fields of `CheetahCudaConfig`. Compositions the
    CUDA backend does not build (routed experts, partial rotary, GELU
    feed-forward) raise instead of resolving to a wrong model."""
    raw = model.raw_config
    _, fam = family_for(raw)
    embed = model.units.get("model.embed_tokens.weight")
    if embed is None or len(embed.shape) != 2:
        raise ValueError("Native backend: units manifest has no embedding tensor.")
    pick = lambda v, d: d if v is None else v  # noqa: E731  (`unwrap_or`)
    hidden = pick(_field_u(raw, "hidden_size"), embed.shape[1])
    vocab = pick(_field_u(raw, "vocab_size"), embed.shape[0])
    layers = pick(_field_u(raw, "num_hidden_layers"), max(model.max_layer_id() + 1, 1))
    q_unit = model.units.get("model.layers.0.self_attn.q_proj.weight")
    k_unit = model.units.get("model.layers.0.self_attn.k_proj.weight")
    if q_unit is None or k_unit is None:
        raise ValueError("Native backend: units manifest has no q_proj / k_proj tensor.")
    q_out, k_out = q_unit.shape[0], k_unit.shape[0]
    gate = model.units.get("model.layers.0.mlp.gate_proj.weight")
    inter = pick(_field_u(raw, "intermediate_size"), gate.shape[0] if gate else 0)
    if not inter:
        raise ValueError("Native backend: cannot resolve the intermediate size from config.json "
                         "or the units manifest.")
    if (_field_u(raw, "num_local_experts") or 0) > 0:
        raise ValueError("CUDA backend: routed-expert (sparse) feed-forward layers are not served.")
    window = (_field_u(raw, "sliding_window") or 0) if pick(_field_b(raw, "use_sliding_window"), True) else 0
    profile = next(((q, kv, hd) for h, v, q, kv, hd in fam["profiles"] if h == hidden and v == vocab), None)
    q_heads = _field_u(raw, "num_attention_heads")
    if q_heads is not None:
        head_dim = pick(_field_u(raw, "head_dim"), profile[2] if profile else q_out // max(q_heads, 1))
        kv_heads = _field_u(raw, "num_key_value_heads")
        if kv_heads is None:
            kv_heads = k_out // head_dim if head_dim and k_out % head_dim == 0 else q_heads
    elif profile is not None:
        q_heads, kv_heads, head_dim = profile
    else:
        raise ValueError(f"Native backend: cannot determine the attention head layout for hidden size "
                         f"{hidden}; provide config.json or extend the family profiles.")
    factor = pick(_field_f(raw, "partial_rotary_factor"), 1.0)
    if factor < 1.0:
        raise ValueError("CUDA backend: partial rotary embeddings are not served.")
    if raw.get("hidden_act") in ("gelu", "gelu_new", "gelu_pytorch_tanh"):
        raise ValueError("CUDA backend: GELU feed-forward layers are not served.")
    tie = pick(_field_b(raw, "tie_word_embeddings"), fam["tie_word_embeddings"])
    if max_positions is None:
        max_positions = pick(_field_u(raw, "max_position_embeddings"), 32768)
        if fam["max_position_embeddings"]:
            max_positions = min(max_positions, fam["max_position_embeddings"])
    return {
        "hidden_size": int(hidden), "num_layers": int(layers), "q_heads": int(q_heads),
        "kv_heads": int(kv_heads), "head_dim": int(head_dim), "rotary_dim": int(head_dim),
        "intermediate_size": int(inter), "vocab_size": int(vocab),
        "rms_eps": float(pick(_field_f(raw, "rms_norm_eps"), fam["rms_norm_eps"])),
        "rope_theta": float(pick(_field_f(raw, "rope_theta"), fam["rope_theta"])),
        "tie_word_embeddings": 1 if tie else 0, "sliding_window": int(window),
        "max_positions": int(max_positions),
    }


SHAPES = {"qwen2-0.5b": QWEN2_0_5B, "qwen2-7b": QWEN2_7B, "tiny": TINY, "tiny-7b-heads": TINY_7B_HEADS,
          "tiny-llama": TINY_LLAMA, "tiny-mistral": TINY_MISTRAL, "tiny-qwen3": TINY_QWEN3,
          "llama-1b": LLAMA_1B}


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
