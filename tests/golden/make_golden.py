"""Generate the committed golden fixtures that pin the CPU oracle's Q2_K / Q3_K / Q4_K / Q5_K /
Q6_K / Q8_0 decode.

The k-quant format is third-party (GGML); fxeqxmulfx/kernite has no implementation of it. The
owner's published Python package gguf-py (version 0.19.0, ``gguf/quants.py``, ``Q2_K``, ``Q3_K``,
``Q4_K``, ``Q5_K``, ``Q6_K`` and ``Q8_0.dequantize_blocks``) is imported here, in the development
container, to dequantise a fixed set of blocks. Its float32 outputs are stored bit for bit in
``kquant_golden.npz`` and the tests compare the oracle (and, on the GPU, the device decode)
against them. The GPU box does not need gguf: only the .npz travels.

Block sets per type:
  * ``gen``: 64 blocks from the oracle's own synthetic generator (stream key of seed 1234,
    tensor 7), the distribution every bench and parity test uses;
  * ``raw``: 64 blocks of uniformly random bytes (any fp16 d/dmin: subnormal, inf, NaN);
  * ``kat``: hand-built known-answer blocks: d = 1.0, dmin = 0, one scale set, quant
    patterns 0..15 / 0..63, every 6-bit scale and min value through the Q4_K packing, every
    4-bit scale and min (Q2_K), every 6-bit Q3_K scale and hmask pattern, every int8 (Q8_0).
Array names start with the type: q2k, q3k, q4k, q5k, q6k, q8_0 (Q8_0 counted in units of eight
34-byte blocks, 256 weights).
Plus a small matvec case (rows 8, K 512, batch 3) with its float64 reference outputs computed
from gguf's float32 weights.

Run:  python tests/golden/make_golden.py   (writes tests/golden/kquant_golden.npz)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import gguf  # noqa: E402  (gguf-py, development container only)
from gguf import GGMLQuantizationType as T  # noqa: E402
from gguf.quants import dequantize  # noqa: E402

import oracle  # noqa: E402


def fp16_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float16).view(np.uint16)[0])


def kat_q4k() -> np.ndarray:
    blocks = []
    # (1) one scale set to 1, the rest 0, quant patterns 0..15 along the block
    for j in range(8):
        b = np.zeros(144, dtype=np.uint8)
        b[0:2] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        b[2:4] = 0
        sc = np.zeros(8, dtype=np.int64)
        sc[j] = 1
        b[4:16] = pack_q4k_scales(sc, np.zeros(8, dtype=np.int64))
        qs = np.array([(i % 16) | (((i + 5) % 16) << 4) for i in range(128)], dtype=np.uint8)
        b[16:] = qs
        blocks.append(b)
    # (2) every 6-bit value of every scale slot and min slot, with d = dmin = 1
    for v in range(64):
        b = np.zeros(144, dtype=np.uint8)
        b[0:2] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        b[2:4] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        sc = np.array([(v + 7 * j) % 64 for j in range(8)])
        mn = np.array([(63 - v + 3 * j) % 64 for j in range(8)])
        b[4:16] = pack_q4k_scales(sc, mn)
        b[16:] = np.uint8(0x5A)
        blocks.append(b)
    return np.concatenate(blocks)


def pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """GGML's 12-byte packing of eight 6-bit scales and mins (the inverse of get_scale_min)."""
    s = np.zeros(12, dtype=np.int64)
    for j in range(4):
        s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        s[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
        s[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
    return s.astype(np.uint8)


def kat_q5k() -> np.ndarray:
    blocks = []
    # one scale set to 1 (d = 1, dmin = 0), nibble and fifth-bit patterns covering q = 0..31
    for j in range(8):
        b = np.zeros(176, dtype=np.uint8)
        b[0:2] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        sc = np.zeros(8, dtype=np.int64)
        sc[j] = 1
        b[4:16] = pack_q4k_scales(sc, np.zeros(8, dtype=np.int64))
        b[16:48] = np.array([(37 * i + 11 * j) % 256 for i in range(32)], dtype=np.uint8)
        b[48:] = np.array([(i % 16) | (((i + 5) % 16) << 4) for i in range(128)], dtype=np.uint8)
        blocks.append(b)
    # every 6-bit value of every scale slot and min slot, d = dmin = 1, all fifth bits set
    for v in range(64):
        b = np.zeros(176, dtype=np.uint8)
        b[0:2] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        b[2:4] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        sc = np.array([(v + 7 * j) % 64 for j in range(8)])
        mn = np.array([(63 - v + 3 * j) % 64 for j in range(8)])
        b[4:16] = pack_q4k_scales(sc, mn)
        b[16:48] = np.uint8(0xFF)
        b[48:] = np.uint8(0x5A)
        blocks.append(b)
    return np.concatenate(blocks)


def kat_q6k() -> np.ndarray:
    blocks = []
    for sgn in (1, -1):
        for rot in range(4):
            b = np.zeros(210, dtype=np.uint8)
            q = np.array([(e + 17 * rot) % 64 for e in range(256)], dtype=np.int64)
            ql = np.zeros(128, dtype=np.int64)
            qh = np.zeros(64, dtype=np.int64)
            for h in range(2):
                for l in range(32):
                    e0, e1, e2, e3 = 128 * h + l, 128 * h + l + 32, 128 * h + l + 64, 128 * h + l + 96
                    ql[64 * h + l] = (q[e0] & 15) | ((q[e2] & 15) << 4)
                    ql[64 * h + l + 32] = (q[e1] & 15) | ((q[e3] & 15) << 4)
                    qh[32 * h + l] = (q[e0] >> 4) | ((q[e1] >> 4) << 2) | ((q[e2] >> 4) << 4) | ((q[e3] >> 4) << 6)
            b[0:128] = ql.astype(np.uint8)
            b[128:192] = qh.astype(np.uint8)
            b[192:208] = np.full(16, sgn, dtype=np.int8).view(np.uint8)
            b[208:210] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
            blocks.append(b)
    # every int8 scale value across the 16 slots
    for base in range(0, 256, 16):
        b = np.zeros(210, dtype=np.uint8)
        b[0:192] = np.uint8(0xA5)
        b[192:208] = np.array([(base + i) % 256 for i in range(16)], dtype=np.uint8)
        b[208:210] = np.array([fp16_bits(0.5)], dtype=np.uint16).view(np.uint8)
        blocks.append(b)
    return np.concatenate(blocks)


def kat_q2k() -> np.ndarray:
    blocks = []
    # every 4-bit scale / min pair across the 16 slots, d = dmin = 1, each crumb pattern
    for base in range(0, 256, 16):
        b = np.zeros(84, dtype=np.uint8)
        b[0:16] = np.array([(base + 17 * i) % 256 for i in range(16)], dtype=np.uint8)
        b[16:80] = np.array([(i * 0x1B) % 256 for i in range(64)], dtype=np.uint8)
        b[80:82] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        b[82:84] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        blocks.append(b)
    # one scale set to 1 (min 0), quants 0..3 along the block, d = 0.5
    for i in range(16):
        b = np.zeros(84, dtype=np.uint8)
        b[i] = 1
        b[16:80] = np.uint8(0b11100100)
        b[80:82] = np.array([fp16_bits(0.5)], dtype=np.uint16).view(np.uint8)
        blocks.append(b)
    return np.concatenate(blocks)


def pack_q3k_scales(sc: np.ndarray) -> np.ndarray:
    """GGML's 12-byte packing of sixteen 6-bit Q3_K scales (values 0..63, stored + 32)."""
    s = np.zeros(12, dtype=np.int64)
    for i in range(16):
        s[i % 8] |= (sc[i] & 15) << (4 * (i // 8))
        s[8 + i % 4] |= ((sc[i] >> 4) & 3) << (2 * (i // 4))
    return s.astype(np.uint8)


def kat_q3k() -> np.ndarray:
    blocks = []
    # every 6-bit stored scale value through the packing, d = 1, alternating hmask bits
    for v in range(0, 64, 4):
        b = np.zeros(110, dtype=np.uint8)
        b[0:32] = np.array([0x55 if i % 2 else 0xAA for i in range(32)], dtype=np.uint8)
        b[32:96] = np.array([(i * 0x2D) % 256 for i in range(64)], dtype=np.uint8)
        b[96:108] = pack_q3k_scales(np.array([(v + i) % 64 for i in range(16)]))
        b[108:110] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
        blocks.append(b)
    # one sub-block scaled by +1 (stored 33), all q values -4..3 via hmask all-0 and all-1
    for i in range(16):
        for hm in (0x00, 0xFF):
            b = np.zeros(110, dtype=np.uint8)
            b[0:32] = np.uint8(hm)
            b[32:96] = np.uint8(0b11100100)
            sc = np.full(16, 32)
            sc[i] = 33
            b[96:108] = pack_q3k_scales(sc)
            b[108:110] = np.array([fp16_bits(1.0)], dtype=np.uint16).view(np.uint8)
            blocks.append(b)
    return np.concatenate(blocks)


def kat_q8_0() -> np.ndarray:
    blocks = []
    # every int8 value (eight per 32-byte block), d = 1, 0.5, -2 and a subnormal
    for d in (1.0, 0.5, -2.0, 2.0 ** -20):
        for base in range(0, 256, 32):
            b = np.zeros(34, dtype=np.uint8)
            b[0:2] = np.array([fp16_bits(d)], dtype=np.uint16).view(np.uint8)
            b[2:34] = np.arange(base, base + 32, dtype=np.int64).astype(np.uint8)
            blocks.append(b)
    return np.concatenate(blocks)  # 32 blocks = 4 units


GGUF_TYPES = {2: T.Q2_K, 3: T.Q3_K, 4: T.Q4_K, 5: T.Q5_K, 6: T.Q6_K, 8: T.Q8_0}
GGUF_BLOCK_BYTES = {2: 84, 3: 110, 4: 144, 5: 176, 6: 210, 8: 34}


def gguf_dequant(qtype: int, raw: np.ndarray) -> np.ndarray:
    arr = raw.reshape(-1, GGUF_BLOCK_BYTES[qtype])
    out = dequantize(arr, GGUF_TYPES[qtype])
    return np.ascontiguousarray(out, dtype=np.float32).reshape(-1)


def main() -> None:
    oracle.build(force=True)  # make: rebuilds the library if a source is newer
    rng = np.random.default_rng(20261201)
    data = {"gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")}
    key = oracle.stream_key(1234, 7)
    # types in the order they were added: each type's random draws follow the earlier ones', so
    # adding a type leaves every existing array as it was
    for qtype in (4, 6, 5, 2, 3, 8):
        pre = oracle.GOLDEN_PREFIX[qtype]
        bb = oracle.block_bytes(qtype)
        gen = oracle.fill(qtype, key, 0, 64)
        raw = rng.integers(0, 256, size=64 * bb, dtype=np.uint8)
        kat = {2: kat_q2k, 3: kat_q3k, 4: kat_q4k, 5: kat_q5k, 6: kat_q6k, 8: kat_q8_0}[qtype]()
        for name, blocks in (("gen", gen), ("raw", raw), ("kat", kat)):
            ref = gguf_dequant(qtype, blocks)
            data[f"{pre}_{name}_blocks"] = blocks
            data[f"{pre}_{name}_f32bits"] = ref.view(np.uint32)
        # small matvec case from generated blocks
        rows, K, batch = 8, 512, 3
        W = oracle.fill(qtype, oracle.stream_key(99, qtype), 0, rows * K // 256)
        x = rng.standard_normal((batch, K), dtype=np.float32)
        w = gguf_dequant(qtype, W).reshape(rows, K).astype(np.float64)
        y = x.astype(np.float64) @ w.T
        bound = np.abs(x.astype(np.float64)[:, None, :] * w[None, :, :]).sum(-1)
        data[f"{pre}_mv_W"] = W
        data[f"{pre}_mv_x"] = x
        data[f"{pre}_mv_y"] = y
        data[f"{pre}_mv_bound"] = bound
    out = os.path.join(HERE, "kquant_golden.npz")
    np.savez_compressed(out, **data)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
