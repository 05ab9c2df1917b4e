"""Host-side mirror of the reference's `ModelForward` boundary over the C-ABI
library (`include/cheetah_cuda.h`), plus thin wrappers of the op entries.

`CudaQwen2` behaves like `Qwen2Native` (`src/chat/registrations/qwen2.rs:600-635`)
behind `ModelForward` (`src/chat/registry.rs:57-85`): `forward(tokens, offset)`
returns the final position's logits, `clear_cache()`, `kv_snapshot()`,
`restore_kv_prefix(snapshot, positions)`, `clone()` (shares weights, empty
KV, `registry.rs:95-117`) and `device_name()`. Errors surface as
`CheetahCudaError` carrying the library's last-error string, the way the Rust
side maps `check_native_result` (`src/native.rs:1860-1870`) to `Err(String)`.

There is no CPU fallback: constructing anything here without the built
library or without a CUDA device raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

from .prepared import PreparedModel, resolve_config

# The in-tree build; CHEETAH_CUDA_LIB selects another build of the same ABI.
LIB_PATH = Path(os.environ.get("CHEETAH_CUDA_LIB") or Path(__file__).resolve().parent / "libcheetah_cuda.so")

KV_BF16, KV_F32 = 0, 1


class CheetahCudaError(RuntimeError):
    pass


class CudaConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_uint32), ("num_layers", C.c_uint32), ("q_heads", C.c_uint32),
        ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("rotary_dim", C.c_uint32),
        ("intermediate_size", C.c_uint32), ("vocab_size", C.c_uint32), ("rms_eps", C.c_float),
        ("rope_theta", C.c_float), ("tie_word_embeddings", C.c_int32),
        ("sliding_window", C.c_uint32), ("max_positions", C.c_uint32),
        ("kv_page_tokens", C.c_uint32), ("kv_pool_tokens", C.c_uint32), ("kv_dtype", C.c_int32),
    ]


class ModelInfo(C.Structure):
    _fields_ = [
        ("weight_bytes", C.c_uint64), ("kv_pool_bytes", C.c_uint64),
        ("kv_pages_total", C.c_uint32), ("kv_pages_free", C.c_uint32),
        ("device", C.c_int32), ("quant", C.c_int32),
        ("persistent_decode", C.c_int32), ("reserved", C.c_int32),
    ]


class Residency(C.Structure):
    _fields_ = [("unit_ids", C.POINTER(C.c_char_p)), ("tiers", C.POINTER(C.c_char_p)), ("count", C.c_size_t)]


class ResidencyInfo(C.Structure):
    _fields_ = [
        ("resident_linear_bytes", C.c_uint64), ("streamed_linear_bytes", C.c_uint64),
        ("staging_bytes", C.c_uint64), ("resident_linears", C.c_uint32), ("streamed_linears", C.c_uint32),
        ("planned", C.c_int32), ("reserved", C.c_int32),
    ]


class DecodeAttentionArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k_pool", C.c_void_p), ("v_pool", C.c_void_p),
        ("kv_dtype", C.c_int32), ("page_table", C.c_void_p), ("max_pages_per_seq", C.c_uint32),
        ("seq_lens", C.c_void_p), ("max_seq_len", C.c_uint32), ("num_pages", C.c_uint32),
        ("page_tokens", C.c_uint32), ("batch", C.c_uint32), ("q_heads", C.c_uint32),
        ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("sliding_window", C.c_uint32),
        ("out", C.c_void_p),
    ]


class PrefillAttentionArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k_pool", C.c_void_p), ("v_pool", C.c_void_p),
        ("page_table", C.c_void_p), ("max_pages", C.c_uint32), ("num_pages", C.c_uint32),
        ("page_tokens", C.c_uint32), ("tokens", C.c_uint32), ("offset", C.c_uint32),
        ("q_heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("sliding_window", C.c_uint32), ("out", C.c_void_p),
    ]


# Every symbol include/cheetah_cuda.h declares, with its ctypes signature.
_P, _S, _I = C.c_void_p, C.c_size_t, C.c_int
SIGNATURES = {
    "cheetah_cuda_last_error": (C.c_char_p, []),
    "cheetah_cuda_abi_version": (_I, []),
    "cheetah_cuda_device_count": (_I, [C.POINTER(C.c_int)]),
    "cheetah_cuda_model_open": (_I, [C.c_char_p, C.POINTER(CudaConfig), C.c_char_p, _I, C.POINTER(_P)]),
    "cheetah_cuda_model_free": (_I, [_P]),
    "cheetah_cuda_model_info": (_I, [_P, C.POINTER(ModelInfo)]),
    "cheetah_cuda_model_open_ex": (_I, [C.c_char_p, C.POINTER(CudaConfig), C.c_char_p, _I, C.POINTER(Residency),
                                        C.POINTER(_P)]),
    "cheetah_cuda_model_page_in_unit": (_I, [_P, C.c_char_p, _I, C.POINTER(_I)]),
    "cheetah_cuda_model_evict_unit": (_I, [_P, C.c_char_p, C.POINTER(_I)]),
    "cheetah_cuda_model_residency": (_I, [_P, C.POINTER(ResidencyInfo)]),
    "cheetah_cuda_seq_new": (_I, [_P, C.POINTER(_P)]),
    "cheetah_cuda_seq_free": (_I, [_P]),
    "cheetah_cuda_seq_clear": (_I, [_P]),
    "cheetah_cuda_seq_positions": (_I, [_P, C.POINTER(_S)]),
    "cheetah_cuda_forward": (_I, [_P, _P, _S, _S, _P]),
    "cheetah_cuda_forward_ex": (_I, [_P, _P, _S, _S, _P, _P]),
    "cheetah_cuda_model_coalesce_stats": (_I, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                                C.POINTER(C.c_uint64)]),
    "cheetah_cuda_forward_batch": (_I, [_P, _P, _P, _P, _S, _P, _P]),
    "cheetah_cuda_forward_batch_greedy": (_I, [_P, _P, _P, _P, _S, _S, _P]),
    "cheetah_cuda_generate_greedy": (_I, [_P, C.c_uint32, _S, _S, _P]),
    "cheetah_cuda_seq_stream": (_I, [_P, C.POINTER(_P)]),
    "cheetah_cuda_model_batch_stream": (_I, [_P, C.POINTER(_P)]),
    "cheetah_cuda_seq_snapshot": (_I, [_P, C.POINTER(_P)]),
    "cheetah_cuda_snapshot_positions": (_I, [_P, C.POINTER(_S)]),
    "cheetah_cuda_seq_restore_prefix": (_I, [_P, _P, _S]),
    "cheetah_cuda_snapshot_free": (_I, [_P]),
    "cheetah_cuda_seq_export_kv": (_I, [_P, _S, _P, _P]),
    "cheetah_cuda_op_gemv_bf16": (_I, [_P, _S, _S, _P, _S, _P, _P]),
    "cheetah_cuda_op_decode_attention": (_I, [C.POINTER(DecodeAttentionArgs), _P]),
    "cheetah_cuda_op_decode_attention_noalloc": (_I, [C.POINTER(DecodeAttentionArgs), _P]),
    "cheetah_cuda_op_prefill_attention": (_I, [C.POINTER(PrefillAttentionArgs), _P]),
    "cheetah_cuda_quant_buffer_bytes": (_I, [C.c_char_p, _S, _S, C.POINTER(_S)]),
    "cheetah_cuda_op_quantize_q8": (_I, [_P, _S, _S, _P, _P]),
    "cheetah_cuda_op_quantize_q4": (_I, [_P, _S, _S, _P, _P]),
    "cheetah_cuda_op_gemv_q8": (_I, [_P, _S, _S, _P, _S, _P, _P]),
    "cheetah_cuda_op_gemv_q4": (_I, [_P, _S, _S, _P, _S, _P, _P]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Load libcheetah_cuda.so (built in-tree by `cheetah_b200.build`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise CheetahCudaError(
                f"{LIB_PATH} is missing: build it with `python -m cheetah_b200.build` "
                "(there is no CPU fallback).")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise CheetahCudaError(lib().cheetah_cuda_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def device_count() -> int:
    n = C.c_int(0)
    _check(lib().cheetah_cuda_device_count(C.byref(n)))
    return n.value


class CudaModel:
    """HBM-resident weights + KV page pool on one device (`model_open`)."""

    def __init__(self, prepared_dir: os.PathLike, quant: str = "bf16", device: int = 0,
                 kv_dtype: str = "bf16", max_positions: Optional[int] = None,
                 kv_pool_tokens: int = 0, kv_page_tokens: int = 0,
                 config: Optional[dict] = None, residency: Optional[dict] = None):
        """`residency`: an Ant plan {unit id: "vram" | "ram" | "disk"}
        (`cheetah_cuda_model_open_ex`); None opens every unit HBM-resident."""
        self.prepared_dir = Path(prepared_dir)
        cfg = dict(config) if config else resolve_config(PreparedModel(self.prepared_dir), max_positions)
        if max_positions:
            cfg["max_positions"] = int(max_positions)
        self.cfg = cfg
        self.quant = quant
        c = CudaConfig(cfg["hidden_size"], cfg["num_layers"], cfg["q_heads"], cfg["kv_heads"],
                       cfg["head_dim"], cfg["rotary_dim"], cfg["intermediate_size"], cfg["vocab_size"],
                       cfg["rms_eps"], cfg["rope_theta"], cfg["tie_word_embeddings"],
                       cfg["sliding_window"], cfg["max_positions"], kv_page_tokens, kv_pool_tokens,
                       KV_F32 if kv_dtype == "f32" else KV_BF16)
        handle = C.c_void_p()
        if residency is None:
            _check(lib().cheetah_cuda_model_open(str(self.prepared_dir).encode(), C.byref(c),
                                                 quant.encode(), device, C.byref(handle)))
        else:
            items = sorted(residency.items())
            ids = (C.c_char_p * max(1, len(items)))(*[k.encode() for k, _ in items])
            tiers = (C.c_char_p * max(1, len(items)))(*[v.encode() for _, v in items])
            plan = Residency(ids, tiers, len(items))
            _check(lib().cheetah_cuda_model_open_ex(str(self.prepared_dir).encode(), C.byref(c), quant.encode(),
                                                    device, C.byref(plan), C.byref(handle)))
        self._h = handle

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def info(self) -> dict:
        info = ModelInfo()
        _check(lib().cheetah_cuda_model_info(self._h, C.byref(info)))
        return {f: getattr(info, f) for f, _ in ModelInfo._fields_}

    def residency(self) -> dict:
        info = ResidencyInfo()
        _check(lib().cheetah_cuda_model_residency(self._h, C.byref(info)))
        return {f: getattr(info, f) for f, _ in ResidencyInfo._fields_}

    def page_in_unit(self, unit_id: str, tier: int = 0) -> bool:
        """`AntTierControl::page_in_unit`: True when the manifest knows the unit."""
        known = C.c_int(0)
        _check(lib().cheetah_cuda_model_page_in_unit(self._h, unit_id.encode(), tier, C.byref(known)))
        return bool(known.value)

    def evict_unit(self, unit_id: str) -> bool:
        """`AntTierControl::evict_unit`: True when the manifest knows the unit."""
        known = C.c_int(0)
        _check(lib().cheetah_cuda_model_evict_unit(self._h, unit_id.encode(), C.byref(known)))
        return bool(known.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cheetah_cuda_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_sequence(self) -> "CudaQwen2":
        return CudaQwen2(self)

    def forward_batch(self, seqs, tokens, offsets, want_logits: bool = False):
        """One decode token for each sequence (`cheetah_cuda_forward_batch`).
        Returns the greedy ids (and the [B, vocab] logits when asked)."""
        B = len(seqs)
        handles = (C.c_void_p * B)(*[s._h.value for s in seqs])
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        o = np.ascontiguousarray(np.asarray(offsets, dtype=np.uint64))
        am = np.zeros(B, dtype=np.uint32)
        logits = np.empty((B, self.cfg["vocab_size"]), dtype=np.float32) if want_logits else None
        _check(lib().cheetah_cuda_forward_batch(self._h, handles, _ptr(t), _ptr(o), B,
                                                _ptr(logits) if want_logits else None, _ptr(am)))
        return (am, logits) if want_logits else am

    def coalesce_stats(self) -> dict:
        """Counters of the batcher behind `forward`: single-token calls,
        calls that ran inside batched steps, batched steps."""
        a, b, c = C.c_uint64(0), C.c_uint64(0), C.c_uint64(0)
        _check(lib().cheetah_cuda_model_coalesce_stats(self._h, C.byref(a), C.byref(b), C.byref(c)))
        return {"calls": a.value, "batched_calls": b.value, "batches": c.value}

    def batch_stream_handle(self) -> int:
        """The stream batched calls run on (0 before the first batched call)."""
        s = C.c_void_p()
        _check(lib().cheetah_cuda_model_batch_stream(self._h, C.byref(s)))
        return s.value or 0

    def forward_batch_greedy(self, seqs, tokens, offsets, steps: int) -> np.ndarray:
        """`steps` greedy tokens for each sequence with no host round trip
        between steps (`cheetah_cuda_forward_batch_greedy`): uint32 [B, steps],
        row b holding the ids generated after tokens[b]."""
        B = len(seqs)
        handles = (C.c_void_p * B)(*[s._h.value for s in seqs])
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        o = np.ascontiguousarray(np.asarray(offsets, dtype=np.uint64))
        out = np.zeros((B, steps), dtype=np.uint32)
        _check(lib().cheetah_cuda_forward_batch_greedy(self._h, handles, _ptr(t), _ptr(o), B, steps, _ptr(out)))
        return out


class CudaSnapshot:
    def __init__(self, handle: C.c_void_p, model: CudaModel):
        self._h = handle
        self._model = model

    @property
    def positions(self) -> int:
        n = C.c_size_t(0)
        _check(lib().cheetah_cuda_snapshot_positions(self._h, C.byref(n)))
        return n.value

    def __del__(self):
        if getattr(self, "_h", None):
            lib().cheetah_cuda_snapshot_free(self._h)
            self._h = None


class CudaQwen2:
    """`ModelForward` over one sequence of a `CudaModel` (`qwen2.rs:600-635`)."""

    def __init__(self, model: CudaModel):
        self.model = model
        self.cfg = model.cfg
        handle = C.c_void_p()
        _check(lib().cheetah_cuda_seq_new(model.handle, C.byref(handle)))
        self._h = handle
        self._logits = np.zeros(self.cfg["vocab_size"], dtype=np.float32)

    @classmethod
    def load(cls, prepared_dir: os.PathLike, **kwargs) -> "CudaQwen2":
        return cls(CudaModel(prepared_dir, **kwargs))

    def device_name(self) -> str:
        return "cuda-b200"

    def clone(self) -> "CudaQwen2":
        """Shares the weights, starts with an empty KV (`registry.rs:95-117`)."""
        return CudaQwen2(self.model)

    def forward(self, tokens: Sequence[int], offset: int, out: Optional[np.ndarray] = None) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        logits = out if out is not None else np.empty(self.cfg["vocab_size"], dtype=np.float32)
        _check(lib().cheetah_cuda_forward(self._h, _ptr(t) if t.size else None, t.size, offset,
                                          _ptr(logits)))
        return logits

    def forward_greedy(self, tokens: Sequence[int], offset: int,
                       logits_out: Optional[np.ndarray] = None) -> int:
        """Forward plus on-device greedy argmax (`engine.rs:2247-2253`)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        am = C.c_uint32(0)
        lp = _ptr(logits_out) if logits_out is not None else None
        _check(lib().cheetah_cuda_forward_ex(self._h, _ptr(t) if t.size else None, t.size, offset,
                                             lp, C.byref(am)))
        return am.value

    def generate_greedy(self, first_token: int, offset: int, steps: int,
                        wait: bool = True) -> Optional[np.ndarray]:
        """Device-resident greedy decode of `steps` tokens (no host round trip
        per token). With wait=False the steps are only enqueued."""
        out = np.zeros(steps, dtype=np.uint32) if wait else None
        _check(lib().cheetah_cuda_generate_greedy(self._h, int(first_token), offset, steps,
                                                  _ptr(out) if wait else None))
        return out

    def stream_handle(self) -> int:
        s = C.c_void_p()
        _check(lib().cheetah_cuda_seq_stream(self._h, C.byref(s)))
        return s.value or 0

    def clear_cache(self) -> None:
        _check(lib().cheetah_cuda_seq_clear(self._h))

    def positions(self) -> int:
        n = C.c_size_t(0)
        _check(lib().cheetah_cuda_seq_positions(self._h, C.byref(n)))
        return n.value

    def kv_snapshot(self) -> CudaSnapshot:
        handle = C.c_void_p()
        _check(lib().cheetah_cuda_seq_snapshot(self._h, C.byref(handle)))
        return CudaSnapshot(handle, self.model)

    def restore_kv_prefix(self, snapshot: CudaSnapshot, positions: int) -> bool:
        _check(lib().cheetah_cuda_seq_restore_prefix(self._h, snapshot._h, positions))
        return True

    def kv_layer(self, layer: int):
        n = self.positions() * self.cfg["kv_heads"] * self.cfg["head_dim"]
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        if n:
            _check(lib().cheetah_cuda_seq_export_kv(self._h, layer, _ptr(k), _ptr(v)))
        return k, v

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cheetah_cuda_seq_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- op entries over torch CUDA tensors (caller-owned device memory) ----

def _stream_ptr(stream) -> Optional[int]:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def gemv_bf16(weight, x, stream=None):
    """y = W . x (`ops.rs:246`). weight: bf16 [rows, cols]; x: f32 [batch, cols]."""
    import torch
    assert weight.dtype == torch.bfloat16 and x.dtype == torch.float32 and weight.is_cuda
    rows, cols = weight.shape
    xb = x.reshape(-1, cols).contiguous()
    y = torch.empty(xb.shape[0], rows, dtype=torch.float32, device=x.device)
    _check(lib().cheetah_cuda_op_gemv_bf16(weight.data_ptr(), rows, cols, xb.data_ptr(),
                                           xb.shape[0], y.data_ptr(), _stream_ptr(stream)))
    return y


def quant_buffer_bytes(fmt: str, rows: int, cols: int) -> int:
    n = C.c_size_t(0)
    _check(lib().cheetah_cuda_quant_buffer_bytes(fmt.encode(), rows, cols, C.byref(n)))
    return n.value


def quantize(weight, fmt: str, stream=None):
    """Per-row q8/q4 quantisation (`q8.rs:91`, `q4.rs:126`) of bf16 [rows, cols]
    on the device; returns the uint8 buffer in the reference layout."""
    import torch
    assert weight.dtype == torch.bfloat16 and weight.is_cuda and weight.is_contiguous()
    rows, cols = weight.shape
    out = torch.empty(quant_buffer_bytes(fmt, rows, cols), dtype=torch.uint8, device=weight.device)
    fn = lib().cheetah_cuda_op_quantize_q8 if fmt == "q8" else lib().cheetah_cuda_op_quantize_q4
    _check(fn(weight.data_ptr(), rows, cols, out.data_ptr(), _stream_ptr(stream)))
    return out


def gemv_quant(buffer, fmt: str, rows: int, cols: int, x, stream=None):
    """y = W . x over a q8/q4 reference-layout buffer (`ops.rs:544`, `:586`)."""
    import torch
    xb = x.reshape(-1, cols).contiguous()
    y = torch.empty(xb.shape[0], rows, dtype=torch.float32, device=x.device)
    fn = lib().cheetah_cuda_op_gemv_q8 if fmt == "q8" else lib().cheetah_cuda_op_gemv_q4
    _check(fn(buffer.data_ptr(), rows, cols, xb.data_ptr(), xb.shape[0], y.data_ptr(), _stream_ptr(stream)))
    return y


def decode_attention(q, k_pool, v_pool, page_table, seq_lens, max_seq_len: int,
                     sliding_window: int = 0, out=None, stream=None, noalloc: bool = False):
    """Paged GQA decode attention (`ops.rs:1357-1467`). noalloc=True takes the
    entry point whose scratch is a fixed array inside the library (for callers
    that cannot let the library allocate device memory).

    q [B, q_heads, D] f32; k_pool/v_pool [pages, kv_heads, page_tokens, D]
    bf16 or f32; page_table [B, max_pages] int32; seq_lens [B] int32."""
    import torch
    B, qh, D = q.shape
    pages, kvh, pt, D2 = k_pool.shape
    assert D == D2 and v_pool.shape == k_pool.shape and page_table.dtype == torch.int32
    if out is None:
        out = torch.empty_like(q)
    args = DecodeAttentionArgs(
        q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        KV_F32 if k_pool.dtype == torch.float32 else KV_BF16,
        page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(), max_seq_len, pages, pt,
        B, qh, kvh, D, sliding_window, out.data_ptr())
    fn = lib().cheetah_cuda_op_decode_attention_noalloc if noalloc else lib().cheetah_cuda_op_decode_attention
    _check(fn(C.byref(args), _stream_ptr(stream)))
    return out


def prefill_attention(q, k_pool, v_pool, page_table, offset: int, sliding_window: int = 0,
                      out=None, stream=None):
    """Causal attention of a prefill chunk (`ops.rs:1357-1421` per query row).

    q [T, q_heads, D] bf16 (RoPE applied) for positions offset .. offset+T-1;
    k_pool/v_pool [pages, kv_heads, page_tokens, D] bf16 holding positions
    0 .. offset+T-1 of the sequence; page_table [max_pages] int32.
    Returns out [T, q_heads, D] bf16."""
    import torch
    T, qh, D = q.shape
    pages, kvh, pt, D2 = k_pool.shape
    assert D == D2 and v_pool.shape == k_pool.shape and page_table.dtype == torch.int32
    assert q.dtype == torch.bfloat16 and k_pool.dtype == torch.bfloat16 and q.is_contiguous()
    if out is None:
        out = torch.empty_like(q)
    args = PrefillAttentionArgs(q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), page_table.data_ptr(),
                                page_table.numel(), pages, pt, T, offset, qh, kvh, D, sliding_window,
                                out.data_ptr())
    _check(lib().cheetah_cuda_op_prefill_attention(C.byref(args), _stream_ptr(stream)))
    return out
