"""TEST INFRASTRUCTURE ONLY: ctypes wrapper over oracle/build/liboracle_cpu.so.

Every function mirrors one reference function (file:line in ref_cpu.h).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "liboracle_cpu.so"

BF16, F16, F32 = 0, 1, 2
QUANT_NONE, QUANT_Q8, QUANT_Q4 = 0, 1, 2
_DTYPES = {"BF16": BF16, "F16": F16, "F32": F32}

_lib: Optional[C.CDLL] = None


def build() -> Path:
    """Compile the oracle (and oracle/_ref when the reference is mounted)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        sources = [HERE / "ref_cpu.cpp", HERE / "ref_cpu.h"]
        if not LIB_PATH.exists() or any(f.stat().st_mtime > LIB_PATH.stat().st_mtime for f in sources):
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


class OracleConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_uint32), ("num_layers", C.c_uint32), ("q_heads", C.c_uint32),
        ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("rotary_dim", C.c_uint32),
        ("intermediate_size", C.c_uint32), ("vocab_size", C.c_uint32), ("rms_eps", C.c_float),
        ("rope_theta", C.c_float), ("tie_word_embeddings", C.c_int32),
        ("sliding_window", C.c_uint32), ("quant", C.c_int32),
    ]


_P = C.c_void_p
_S = C.c_size_t


def _declare(l: C.CDLL) -> None:
    sig = {
        "oracle_set_threads": (None, [C.c_int]),
        "oracle_get_threads": (C.c_int, []),
        "oracle_has_avx2": (C.c_int, []),
        "oracle_gemv": (None, [_P, C.c_int, _S, _S, _P, _P]),
        "oracle_gemm": (None, [_P, C.c_int, _S, _S, _P, _S, _P]),
        "oracle_gemv_q8": (None, [_P, _S, _S, _P, _P]),
        "oracle_gemv_q4": (None, [_P, _S, _S, _P, _P]),
        "oracle_q8_row_bytes": (_S, [_S]),
        "oracle_q4_row_bytes": (_S, [_S]),
        "oracle_q8_bytes": (_S, [_S, _S]),
        "oracle_q4_bytes": (_S, [_S, _S]),
        "oracle_quantize_q8": (C.c_int, [_P, _S, _S, _P]),
        "oracle_quantize_q4": (C.c_int, [_P, _S, _S, _P]),
        "oracle_q8_dequant": (C.c_float, [_P, _S, _S, _S, _S]),
        "oracle_q4_dequant": (C.c_float, [_P, _S, _S, _S, _S]),
        "oracle_rmsnorm": (None, [_P, _S, _P, C.c_int, C.c_float]),
        "oracle_rope_in_place": (None, [_P, _S, _S, _S, C.c_float]),
        "oracle_rope_heads": (None, [_P, _S, _S, _S, _S, C.c_float]),
        "oracle_silu_multiply": (None, [_P, _P, _S]),
        "oracle_softmax": (None, [_P, _S]),
        "oracle_attention": (None, [_P, _P, _S, _S, _P, _S, _S, _S, _S, _P]),
        "oracle_model_new": (_P, [C.POINTER(OracleConfig)]),
        "oracle_model_free": (None, [_P]),
        "oracle_model_set_unit": (C.c_int, [_P, C.c_char_p, _P, C.c_int, _S]),
        "oracle_model_prepare": (C.c_int, [_P]),
        "oracle_model_forward": (C.c_int, [_P, _P, _S, _S, _S, _P]),
        "oracle_model_clear": (None, [_P]),
        "oracle_model_positions": (_S, [_P]),
        "oracle_model_kv_export": (C.c_int, [_P, _S, _P, _P]),
        "oracle_model_kv_restore": (C.c_int, [_P, _S, _P, _P]),
        "oracle_model_hidden": (C.c_int, [_P, _P]),
        "oracle_last_error": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be contiguous"
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return lib().oracle_get_threads()


def gemv(weight: np.ndarray, rows: int, cols: int, x: np.ndarray, dtype: int = BF16) -> np.ndarray:
    """ops.rs:246 gemv. weight: raw bytes or typed array of the stored dtype."""
    w = np.ascontiguousarray(weight)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().oracle_gemv(_ptr(w), dtype, rows, cols, _ptr(x), _ptr(y))
    return y


def gemm(weight: np.ndarray, rows: int, cols: int, x: np.ndarray, dtype: int = BF16) -> np.ndarray:
    """ops.rs:308 gemm: x [n, cols] -> y [n, rows]."""
    w = np.ascontiguousarray(weight)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size // cols
    y = np.zeros((n, rows), dtype=np.float32)
    lib().oracle_gemm(_ptr(w), dtype, rows, cols, _ptr(x), n, _ptr(y))
    return y


def q8_bytes(rows: int, cols: int) -> int:
    return lib().oracle_q8_bytes(rows, cols)


def q4_bytes(rows: int, cols: int) -> int:
    return lib().oracle_q4_bytes(rows, cols)


def q8_row_bytes(cols: int) -> int:
    return lib().oracle_q8_row_bytes(cols)


def q4_row_bytes(cols: int) -> int:
    return lib().oracle_q4_row_bytes(cols)


def quantize_q8(values: np.ndarray, rows: int, cols: int) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.size != rows * cols:
        raise ValueError(f"Q8 quantization expected {rows * cols} elements, found {v.size}.")
    out = np.zeros(q8_bytes(rows, cols), dtype=np.uint8)
    lib().oracle_quantize_q8(_ptr(v), rows, cols, _ptr(out))
    return out


def quantize_q4(values: np.ndarray, rows: int, cols: int) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.size != rows * cols:
        raise ValueError(f"Q4 quantization expected {rows * cols} elements, found {v.size}.")
    out = np.zeros(q4_bytes(rows, cols), dtype=np.uint8)
    lib().oracle_quantize_q4(_ptr(v), rows, cols, _ptr(out))
    return out


def gemv_q8(buffer: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(buffer, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().oracle_gemv_q8(_ptr(b), rows, cols, _ptr(x), _ptr(y))
    return y


def gemv_q4(buffer: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(buffer, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().oracle_gemv_q4(_ptr(b), rows, cols, _ptr(x), _ptr(y))
    return y


def q8_dequant(buffer: np.ndarray, rows: int, cols: int, row: int, col: int) -> float:
    b = np.ascontiguousarray(buffer, dtype=np.uint8)
    return lib().oracle_q8_dequant(_ptr(b), rows, cols, row, col)


def q4_dequant(buffer: np.ndarray, rows: int, cols: int, row: int, col: int) -> float:
    b = np.ascontiguousarray(buffer, dtype=np.uint8)
    return lib().oracle_q4_dequant(_ptr(b), rows, cols, row, col)


def dequant_matrix(buffer: np.ndarray, rows: int, cols: int, fmt: str) -> np.ndarray:
    """Vectorised restatement of the q8/q4 unpacking (`q8.rs:66`, `q4.rs:59-66`),
    checked against the scalar oracle functions in the tests."""
    b = np.ascontiguousarray(buffer, dtype=np.uint8)
    scales = b[: rows * 4].view(np.float32)
    if fmt == "q8":
        rb = q8_row_bytes(cols)
        codes = b[rows * 4:].reshape(rows, rb)[:, :cols].view(np.int8).astype(np.float32)
    else:
        rb = q4_row_bytes(cols)
        payload = b[rows * 4:].reshape(rows, rb)
        cols_idx = np.arange(cols)
        bytes_ = payload[:, cols_idx // 2]
        nib = np.where(cols_idx % 2 == 0, bytes_ & 0x0F, bytes_ >> 4).astype(np.int16)
        codes = np.where(nib >= 8, nib - 16, nib).astype(np.float32)
    return (scales[:, None] * codes).astype(np.float32)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: int = BF16) -> np.ndarray:
    out = np.array(x, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(weight)
    lib().oracle_rmsnorm(_ptr(out), out.size, _ptr(w), dtype, eps)
    return out


def rope_in_place(values: np.ndarray, heads: int, head_dim: int, position: int, theta: float) -> np.ndarray:
    out = np.array(values, dtype=np.float32, copy=True)
    lib().oracle_rope_in_place(_ptr(out), heads, head_dim, position, theta)
    return out


def rope_heads(values: np.ndarray, heads: int, head_dim: int, rotary_dim: int, position: int,
               theta: float) -> np.ndarray:
    out = np.array(values, dtype=np.float32, copy=True)
    lib().oracle_rope_heads(_ptr(out), heads, head_dim, rotary_dim, position, theta)
    return out


def silu_multiply(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.array(gate, dtype=np.float32, copy=True)
    u = np.ascontiguousarray(up, dtype=np.float32)
    lib().oracle_silu_multiply(_ptr(g), _ptr(u), g.size)
    return g


def softmax(scores: np.ndarray) -> np.ndarray:
    s = np.array(scores, dtype=np.float32, copy=True)
    lib().oracle_softmax(_ptr(s), s.size)
    return s


def attention(keys: np.ndarray, values: np.ndarray, q: np.ndarray, q_heads: int, kv_heads: int,
              head_dim: int, position: Optional[int] = None, sliding_window: int = 0) -> np.ndarray:
    """ops.rs:1357 GQA attention of one query over an f32 cache [L, kv_heads*head_dim]."""
    k = np.ascontiguousarray(keys, dtype=np.float32)
    v = np.ascontiguousarray(values, dtype=np.float32)
    qq = np.ascontiguousarray(q, dtype=np.float32)
    cache_len = k.size // (kv_heads * head_dim)
    pos = cache_len - 1 if position is None else position
    out = np.zeros(q_heads * head_dim, dtype=np.float32)
    lib().oracle_attention(_ptr(k), _ptr(v), cache_len, pos, _ptr(qq), q_heads, kv_heads,
                           head_dim, sliding_window, _ptr(out))
    return out


class OracleModel:
    """Qwen2Native (`qwen2.rs:92-635`) over a prepared directory."""

    def __init__(self, prepared, cfg: dict, quant: str = "bf16"):
        self._prepared = prepared  # keeps the memmaps alive
        self.cfg = dict(cfg)
        c = OracleConfig(
            cfg["hidden_size"], cfg["num_layers"], cfg["q_heads"], cfg["kv_heads"],
            cfg["head_dim"], cfg["rotary_dim"], cfg["intermediate_size"], cfg["vocab_size"],
            cfg["rms_eps"], cfg["rope_theta"], cfg["tie_word_embeddings"],
            cfg["sliding_window"], {"bf16": QUANT_NONE, "q8": QUANT_Q8, "q4": QUANT_Q4}[quant])
        self._h = lib().oracle_model_new(C.byref(c))
        self._keep = []
        for unit in prepared.units.values():
            if unit.dtype not in _DTYPES:
                continue
            data = np.ascontiguousarray(unit.data)
            self._keep.append(data)
            lib().oracle_model_set_unit(self._h, unit.unit_id.encode(), _ptr(data),
                                        _DTYPES[unit.dtype], data.nbytes)
        if lib().oracle_model_prepare(self._h) != 0:
            raise RuntimeError(lib().oracle_last_error().decode())

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().oracle_model_free(h)
            self._h = None

    def forward(self, tokens: Sequence[int], offset: int, chunk_rows: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.zeros(self.cfg["vocab_size"], dtype=np.float32)
        rc = lib().oracle_model_forward(self._h, _ptr(t) if t.size else None, t.size, offset,
                                        chunk_rows, _ptr(logits))
        if rc != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        return logits

    def clear_cache(self) -> None:
        lib().oracle_model_clear(self._h)

    def positions(self) -> int:
        return lib().oracle_model_positions(self._h)

    def kv_layer(self, layer: int):
        n = self.positions() * self.cfg["kv_heads"] * self.cfg["head_dim"]
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        lib().oracle_model_kv_export(self._h, layer, _ptr(k), _ptr(v))
        return k, v

    def kv_snapshot(self):
        return self.positions(), [self.kv_layer(i) for i in range(self.cfg["num_layers"])]

    def restore_kv_prefix(self, snapshot, positions: int) -> None:
        total, layers = snapshot
        keep = min(positions, total)
        ks = [np.ascontiguousarray(k) for k, _ in layers]
        vs = [np.ascontiguousarray(v) for _, v in layers]
        kp = (C.c_void_p * len(ks))(*[_ptr(k) for k in ks])
        vp = (C.c_void_p * len(vs))(*[_ptr(v) for v in vs])
        lib().oracle_model_kv_restore(self._h, keep, kp, vp)

    def hidden(self) -> np.ndarray:
        out = np.zeros(self.cfg["hidden_size"], dtype=np.float32)
        lib().oracle_model_hidden(self._h, _ptr(out))
        return out
