"""ctypes binding of the CPU oracle (kq_oracle.c) and the CPU baseline (kq_cpu.c).

TEST INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline
leg import this module, as the checker or as the timed CPU baseline; the product path
(``kernite_b200``, ``libkq.so``) never does.

The k-quant path does not exist in fxeqxmulfx/kernite. The oracle restates the GGML k-quant
format; it is pinned against gguf-py 0.19.0's numpy dequantizer (``gguf/quants.py``,
``Q2_K``, ``Q3_K``, ``Q4_K``, ``Q5_K``, ``Q6_K`` and ``Q8_0.dequantize_blocks``) through the
fixtures in
``tests/golden/``, and its fp16 decode against kernite's table in
``crates/cuda/src/half.rs:165-180``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

Q4K_BYTES = 144
Q6K_BYTES = 210
Q5K_BYTES = 176
Q2K_BYTES = 84
Q3K_BYTES = 110
Q8_0_UNIT_BYTES = 272  # eight 34-byte Q8_0 blocks = 256 weights
QK = 256
# type numbers of the oracle: k-quants by their bit width, Q8_0 as 8
UNIT_BYTES = {2: Q2K_BYTES, 3: Q3K_BYTES, 4: Q4K_BYTES, 5: Q5K_BYTES, 6: Q6K_BYTES,
              8: Q8_0_UNIT_BYTES}
# names of the fixture arrays' prefixes in tests/golden/kquant_golden.npz
GOLDEN_PREFIX = {2: "q2k", 3: "q3k", 4: "q4k", 5: "q5k", 6: "q6k", 8: "q8_0"}

_lib = None


def build(force: bool = False) -> str:
    """Compile oracle/liboracle.so with make (gcc). Returns the library path."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        f32p = ctypes.POINTER(ctypes.c_float)
        f64p = ctypes.POINTER(ctypes.c_double)
        L.kqo_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.kqo_fp16_to_f32.restype = ctypes.c_float
        L.kqo_f32_to_fp16.argtypes = [ctypes.c_float]
        L.kqo_f32_to_fp16.restype = ctypes.c_uint16
        L.kqo_q4k_scale_min.argtypes = [u8p, ctypes.c_int, u8p, u8p]
        L.kqo_q4k_scale_min.restype = None
        for name in ("kqo_dequant_q4k", "kqo_dequant_q5k", "kqo_dequant_q6k", "kqo_dequant_q2k",
                     "kqo_dequant_q3k", "kqo_dequant_q8_0"):
            fn = getattr(L, name)
            fn.argtypes = [u8p, ctypes.c_size_t, f32p]
            fn.restype = None
        L.kqo_dequant.argtypes = [ctypes.c_int, u8p, ctypes.c_size_t, f32p]
        L.kqo_dequant.restype = ctypes.c_int
        L.kqo_q3k_scale.argtypes = [u8p, ctypes.c_int]
        L.kqo_q3k_scale.restype = ctypes.c_int
        L.kqo_matvec_ref.argtypes = [
            ctypes.c_int, u8p, f32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
            ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64, f64p, f64p,
        ]
        L.kqo_matvec_ref.restype = None
        for name in ("kqo_fill_q4k", "kqo_fill_q5k", "kqo_fill_q6k", "kqo_fill_q2k", "kqo_fill_q3k",
                     "kqo_fill_q8_0"):
            fn = getattr(L, name)
            fn.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
            fn.restype = None
        L.kqo_stream_key.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.kqo_stream_key.restype = ctypes.c_uint64
        L.kqo_splitmix_at.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.kqo_splitmix_at.restype = ctypes.c_uint64
        L.kqo_matvec_cpu.argtypes = [
            ctypes.c_int, u8p, f32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, f32p,
            ctypes.c_int,
        ]
        L.kqo_matvec_cpu.restype = ctypes.c_int
        _lib = L
    return _lib


def _u8(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _f32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f64(a: np.ndarray):
    assert a.dtype == np.float64 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def block_bytes(qtype: int) -> int:
    """Bytes per 256 weights (one super-block; for Q8_0, eight blocks)."""
    return UNIT_BYTES[qtype]


def fp16_to_f32(h: int) -> float:
    return lib().kqo_fp16_to_f32(h)


def f32_to_fp16(x: float) -> int:
    return lib().kqo_f32_to_fp16(x)


def q3k_scale(scales12: bytes, i: int) -> int:
    """Scale i (0..15) of a Q3_K block's 12 packed scale bytes, minus 32."""
    buf = np.frombuffer(bytes(scales12), dtype=np.uint8).copy()
    return lib().kqo_q3k_scale(_u8(buf), i)


def q4k_scale_min(scales12: bytes, j: int) -> tuple[int, int]:
    buf = np.frombuffer(bytes(scales12), dtype=np.uint8).copy()
    sc = ctypes.c_uint8()
    m = ctypes.c_uint8()
    lib().kqo_q4k_scale_min(_u8(buf), j, ctypes.byref(sc), ctypes.byref(m))
    return sc.value, m.value


def dequant(qtype: int, blocks: np.ndarray) -> np.ndarray:
    """Dequantise raw block bytes (uint8, n*BLK) into n*256 float32, canonical order."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    n = blocks.size // block_bytes(qtype)
    assert n * block_bytes(qtype) == blocks.size
    out = np.empty(n * QK, dtype=np.float32)
    if lib().kqo_dequant(qtype, _u8(blocks), n, _f32(out)) != 0:
        raise ValueError(f"unknown type {qtype}")
    return out


def stream_key(seed: int, tensor: int) -> int:
    return lib().kqo_stream_key(seed & (2**64 - 1), tensor & (2**64 - 1))


def splitmix_at(key: int, i: int) -> int:
    return lib().kqo_splitmix_at(key, i)


def fill(qtype: int, key: int, b0: int, n: int) -> np.ndarray:
    """Blocks [b0, b0+n) of the synthetic tensor with stream key `key`, as raw bytes."""
    out = np.empty(n * block_bytes(qtype), dtype=np.uint8)
    fn = {2: lib().kqo_fill_q2k, 3: lib().kqo_fill_q3k, 4: lib().kqo_fill_q4k,
          5: lib().kqo_fill_q5k, 6: lib().kqo_fill_q6k, 8: lib().kqo_fill_q8_0}[qtype]
    fn(_u8(out), key, b0, n)
    return out


def matvec_ref(qtype: int, W: np.ndarray, x: np.ndarray, K: int, r0: int, r1: int):
    """Reference y and bound (f64) for rows [r0, r1) of W (raw bytes holding all rows from 0)
    against x of shape (batch, K). Returns arrays of shape (batch, r1 - r0)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    batch = x.shape[0]
    assert x.shape[1] == K
    W = np.ascontiguousarray(W, dtype=np.uint8).reshape(-1)
    rows_alloc = r1  # outputs indexed by absolute row
    y = np.zeros(batch * rows_alloc, dtype=np.float64)
    bound = np.zeros(batch * rows_alloc, dtype=np.float64)
    lib().kqo_matvec_ref(qtype, _u8(W), _f32(x), K, r0, r1, batch, K, rows_alloc, _f64(y), _f64(bound))
    y = y.reshape(batch, rows_alloc)[:, r0:r1]
    bound = bound.reshape(batch, rows_alloc)[:, r0:r1]
    return y, bound


def matvec_cpu(qtype: int, W: np.ndarray, x: np.ndarray, rows: int, K: int, threads: int = 1) -> np.ndarray:
    """The AVX2 CPU baseline: y of shape (batch, rows), f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    batch = x.shape[0]
    y = np.empty(batch * rows, dtype=np.float32)
    rc = lib().kqo_matvec_cpu(qtype, _u8(np.ascontiguousarray(W).reshape(-1)), _f32(x), rows, K, batch, _f32(y), threads)
    if rc != 0:
        raise ValueError(f"kqo_matvec_cpu failed: {rc}")
    return y.reshape(batch, rows)


def cpu_threads() -> int:
    """Host threads available to this process (the CPU baseline uses all of them)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ---------------------------------------------------------------- a decode step's attention

def rope_ref(qkv: np.ndarray, nh: int, nkv: int, d: int, pos: int, base: float):
    """The step's q and k heads rotated by position `pos` (element pairs (2i, 2i+1) by the angle
    pos * base^(-2i/d), GGML's "norm" rotary mode), and v, in f64: (q (nh, d), k (nkv, d),
    v (nkv, d)). kernite has no RoPE; this is the published rotary embedding (Su et al., RoFormer)
    in the pairing GGML's Llama uses."""
    x = np.asarray(qkv, dtype=np.float64)
    q = x[: nh * d].reshape(nh, d)
    k = x[nh * d:(nh + nkv) * d].reshape(nkv, d)
    v = x[(nh + nkv) * d:(nh + 2 * nkv) * d].reshape(nkv, d)
    ang = pos * base ** (-2.0 * np.arange(d // 2) / d)
    c, s = np.cos(ang), np.sin(ang)

    def rot(a):
        out = np.empty_like(a)
        out[:, 0::2] = a[:, 0::2] * c - a[:, 1::2] * s
        out[:, 1::2] = a[:, 0::2] * s + a[:, 1::2] * c
        return out

    return rot(q), rot(k), v


def attention_ref(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, nh: int, nkv: int,
                  d: int, length: int):
    """Grouped-query attention of one step's queries q (nh, d) over the first `length` positions
    of the caches (positions, nkv, d), in f64; query head h reads key/value head h // (nh / nkv).
    Returns (out (nh, d), bound (nh, d) = sum_p w_hp |v_p|, the scale of the tolerance). Follows
    kernite's microgpt attention (examples/microgpt/src/gpu.rs:130-230): logits q.k scaled, their
    maximum, exponentials and sum, the weights, the values they weigh."""
    q = np.asarray(q, dtype=np.float64).reshape(nh, d)
    K = np.asarray(k_cache, dtype=np.float64)[:length]
    V = np.asarray(v_cache, dtype=np.float64)[:length]
    grp = nh // nkv
    out = np.zeros((nh, d))
    bound = np.zeros((nh, d))
    for h in range(nh):
        g = h // grp
        logits = K[:, g, :] @ q[h] / np.sqrt(d)
        w = np.exp(logits - logits.max())
        w /= w.sum()
        out[h] = w @ V[:, g, :]
        bound[h] = w @ np.abs(V[:, g, :])
    return out, bound

