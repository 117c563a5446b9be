"""The CPU oracle, pinned before it is trusted.

* fp16 decode: kernite's IEEE table (crates/cuda/src/half.rs:165-180) and its tie/overflow
  cases (half.rs:183-200), then all 65536 encodings against numpy's exact widening.
* Q4_K / Q6_K decode: bit for bit against gguf-py 0.19.0's dequantizer through the committed
  fixtures (tests/golden/kquant_golden.npz, made by tests/golden/make_golden.py).
* Known-answer blocks built by hand (nibble order, scale packing, q - 32).
* The generator's distributions, and the CPU baseline against the f64 reference.
"""
import numpy as np
import pytest

import oracle

# crates/cuda/src/half.rs:167-176
HALF_TABLE = [
    (0x3C00, 1.0), (0xC000, -2.0), (0x7BFF, 65504.0), (0x0400, 6.1035156e-5),
    (0x0001, 5.9604645e-8), (0x03FF, 6.097555e-5), (0x7C00, float("inf")), (0x8000, -0.0),
]


def f32bits(x: float) -> int:
    return int(np.array([x], dtype=np.float32).view(np.uint32)[0])


def test_fp16_table_from_kernite():
    for bits, val in HALF_TABLE:
        assert f32bits(oracle.fp16_to_f32(bits)) == f32bits(val), hex(bits)
        assert oracle.f32_to_fp16(val) == bits, val


def test_fp16_ties_and_overflow_from_kernite():
    two = np.float32(2.0)
    assert oracle.f32_to_fp16(float(np.float32(1.0) + two ** -11)) == 0x3C00
    assert oracle.f32_to_fp16(float(np.float32(1.0) + 3 * two ** -11)) == 0x3C02
    assert oracle.f32_to_fp16(65519.0) == 0x7BFF
    assert oracle.f32_to_fp16(65520.0) == 0x7C00
    assert oracle.f32_to_fp16(float(two ** -25)) == 0
    nxt = np.array([f32bits(float(two ** -25)) + 1], dtype=np.uint32).view(np.float32)[0]
    assert oracle.f32_to_fp16(float(nxt)) == 1


def test_fp16_every_encoding_widens_exactly():
    L = oracle.lib()
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([L.kqo_fp16_to_f32(int(v)) for v in h], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])


def test_f32_to_fp16_matches_numpy_rounding():
    rng = np.random.default_rng(5)
    xs = np.concatenate([
        rng.uniform(2.0 ** -12, 2.0 ** -6, 20000).astype(np.float32),
        (rng.standard_normal(20000) * 1000).astype(np.float32),
        rng.uniform(0, 2.0 ** -14, 5000).astype(np.float32),  # subnormal range
    ])
    want = xs.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_fp16(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(got, want)


ALL_TYPES = [2, 3, 4, 5, 6, 8]  # Q2_K .. Q6_K, Q8_0


@pytest.mark.parametrize("qtype", ALL_TYPES)
@pytest.mark.parametrize("which", ["gen", "raw", "kat"])
def test_dequant_matches_gguf_bit_for_bit(golden, qtype, which):
    pre = oracle.GOLDEN_PREFIX[qtype]
    blocks = golden[f"{pre}_{which}_blocks"]
    want = golden[f"{pre}_{which}_f32bits"]
    got = oracle.dequant(qtype, blocks).view(np.uint32)
    wf, gf = want.view(np.float32), got.view(np.float32)
    nan = np.isnan(wf)
    assert np.array_equal(np.isnan(gf), nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_matvec_ref_matches_golden(golden, qtype):
    pre = oracle.GOLDEN_PREFIX[qtype]
    W = golden[f"{pre}_mv_W"]
    x = golden[f"{pre}_mv_x"]
    y, bound = oracle.matvec_ref(qtype, W, x, 512, 0, 8)
    np.testing.assert_allclose(y, golden[f"{pre}_mv_y"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(bound, golden[f"{pre}_mv_bound"], rtol=1e-12)


def test_q4k_scale_packing_every_value():
    # all 64 values in every slot: bytes packed as GGML does, unpacked by the oracle
    for v in range(64):
        sc = [(v + 7 * j) % 64 for j in range(8)]
        mn = [(63 - v + 3 * j) % 64 for j in range(8)]
        s = [0] * 12
        for j in range(4):
            s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
            s[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
            s[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
        for j in range(8):
            assert oracle.q4k_scale_min(bytes(s), j) == (sc[j], mn[j])


def test_q4k_known_answer_nibble_order():
    # d = 1, dmin = 0, only sub-block j scaled by 1: weights there are the nibbles, in GGML order
    for j in range(8):
        b = np.zeros(144, dtype=np.uint8)
        b[0:2] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
        sc = [0] * 8
        sc[j] = 1
        s = [0] * 12
        for i in range(4):
            s[i] = sc[i] | ((sc[i + 4] >> 4) << 6)
            s[i + 8] = sc[i + 4] & 15
        b[4:16] = s
        qs = np.array([(i % 16) | (((i + 5) % 16) << 4) for i in range(128)], dtype=np.uint8)
        b[16:] = qs
        w = oracle.dequant(4, b)
        c, hi = j // 2, j % 2
        want = np.zeros(256, dtype=np.float32)
        for l in range(32):
            byte = int(qs[32 * c + l])
            want[32 * j + l] = (byte >> 4) if hi else (byte & 15)
        assert np.array_equal(w, want), j


def test_q6k_known_answer_q_minus_32():
    # scale +-1, d = 1: w = +-(q - 32) with q covering 0..63 in the documented positions
    for sgn in (1, -1):
        q = np.array([(e * 5 + 3) % 64 for e in range(256)])
        ql = np.zeros(128, dtype=np.int64)
        qh = np.zeros(64, dtype=np.int64)
        for h in range(2):
            for l in range(32):
                e = [128 * h + l + 32 * g for g in range(4)]
                ql[64 * h + l] = (q[e[0]] & 15) | ((q[e[2]] & 15) << 4)
                ql[64 * h + l + 32] = (q[e[1]] & 15) | ((q[e[3]] & 15) << 4)
                qh[32 * h + l] = sum(((q[e[g]] >> 4) & 3) << (2 * g) for g in range(4))
        b = np.zeros(210, dtype=np.uint8)
        b[:128] = ql
        b[128:192] = qh
        b[192:208] = np.full(16, sgn, dtype=np.int8).view(np.uint8)
        b[208:210] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
        assert np.array_equal(oracle.dequant(6, b), (sgn * (q - 32)).astype(np.float32))


def test_generator_is_counter_based_and_in_range():
    key = oracle.stream_key(42, 3)
    whole = oracle.fill(4, key, 0, 40)
    part = oracle.fill(4, key, 17, 5)
    assert np.array_equal(whole[17 * 144:22 * 144], part)
    blocks = whole.reshape(40, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    dm = blocks[:, 2:4].copy().view(np.float16).astype(np.float32).ravel()
    assert (d >= 2.0 ** -10).all() and (d <= 2.0 ** -6).all()
    assert (dm >= 2.0 ** -10).all() and (dm <= 2.0 ** -6).all()
    w6 = oracle.fill(6, oracle.stream_key(42, 4), 0, 300).reshape(300, 210)
    sc = w6[:, 192:208].copy().view(np.int8)
    assert sc.min() >= -64 and sc.max() <= 63 and sc.min() < -50 and sc.max() > 50
    d6 = w6[:, 208:210].copy().view(np.float16).astype(np.float32)
    assert (d6 >= 2.0 ** -12).all() and (d6 <= 2.0 ** -8).all()
    assert oracle.stream_key(42, 3) != oracle.stream_key(42, 4)


@pytest.mark.parametrize("qtype,K", [(2, 4096), (2, 11008), (3, 4096), (3, 11008), (4, 4096), (5, 4096),
                                     (5, 11008), (6, 4096), (6, 11008), (8, 4096), (8, 11008)])
def test_cpu_baseline_within_tolerance(qtype, K):
    rows = 64
    W = oracle.fill(qtype, oracle.stream_key(7, qtype), 0, rows * K // 256)
    x = np.random.default_rng(1).standard_normal((2, K), dtype=np.float32)
    y_ref, bound = oracle.matvec_ref(qtype, W, x, K, 0, rows)
    y = oracle.matvec_cpu(qtype, W, x, rows, K, threads=3)
    assert (np.abs(y - y_ref) <= 1e-3 * bound).all()


def test_q3k_scale_packing_every_value():
    # sixteen 6-bit scales packed as GGML does (low nibbles in bytes 0-7, high pairs in 8-11)
    for v in range(64):
        sc = [(v + 5 * i) % 64 for i in range(16)]
        s = [0] * 12
        for i in range(16):
            s[i % 8] |= (sc[i] & 15) << (4 * (i // 8))
            s[8 + i % 4] |= ((sc[i] >> 4) & 3) << (2 * (i // 4))
        for i in range(16):
            assert oracle.q3k_scale(bytes(s), i) == sc[i] - 32


def test_q2k_q3k_known_answer_element_order():
    # Q2_K: d = 1, dmin = 0, only sub-block i scaled by 1: its weights are the crumbs of qs in
    # GGML order (element 128h + 32s + l = bits 2s.. of qs[32h + l])
    rng = np.random.default_rng(3)
    qs = rng.integers(0, 256, size=64, dtype=np.uint8)
    hm = rng.integers(0, 256, size=32, dtype=np.uint8)
    want_q2 = np.array([(qs[32 * (e // 128) + e % 32] >> (2 * ((e // 32) % 4))) & 3
                        for e in range(256)], dtype=np.float32)
    for i in range(16):
        b = np.zeros(84, dtype=np.uint8)
        b[i] = 1
        b[16:80] = qs
        b[80:82] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
        w = oracle.dequant(2, b)
        want = np.zeros(256, dtype=np.float32)
        want[16 * i:16 * i + 16] = want_q2[16 * i:16 * i + 16]
        assert np.array_equal(w, want), i
    # Q3_K: every stored scale 33 (scale +1), d = 1: w = low crumb - 4 * (1 - hmask bit)
    b = np.zeros(110, dtype=np.uint8)
    b[0:32] = hm
    b[32:96] = qs
    s = [0] * 12
    for i in range(16):
        s[i % 8] |= (33 & 15) << (4 * (i // 8))
        s[8 + i % 4] |= ((33 >> 4) & 3) << (2 * (i // 4))
    b[96:108] = s
    b[108:110] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
    hbit = np.array([(hm[e % 32] >> (e // 32)) & 1 for e in range(256)])
    assert np.array_equal(oracle.dequant(3, b), (want_q2 - 4 * (1 - hbit)).astype(np.float32))


def test_q8_0_units_are_eight_blocks():
    # a unit of 272 bytes is eight 34-byte blocks, each w = q * d with its own d
    key = oracle.stream_key(5, 8)
    u = oracle.fill(8, key, 0, 3)
    assert u.size == 3 * 272
    blocks = u.reshape(24, 34)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, 2:].view(np.int8).astype(np.float32)
    assert np.array_equal(oracle.dequant(8, u), (q * d).reshape(-1))
    assert (d >= 2.0 ** -12).all() and (d <= 2.0 ** -8).all()
    # counter-based: units 1..2 on their own are the same bytes
    assert np.array_equal(oracle.fill(8, key, 1, 2), u[272:])


@pytest.mark.parametrize("qtype", [2, 3])
def test_new_generators_are_counter_based(qtype):
    key = oracle.stream_key(42, qtype)
    bb = oracle.block_bytes(qtype)
    whole = oracle.fill(qtype, key, 0, 30)
    assert np.array_equal(whole[11 * bb:16 * bb], oracle.fill(qtype, key, 11, 5))
    blocks = whole.reshape(30, bb)
    at = 80 if qtype == 2 else 108
    d = blocks[:, at:at + 2].copy().view(np.float16).astype(np.float32)
    lo, hi = (2.0 ** -9, 2.0 ** -5) if qtype == 2 else (2.0 ** -11, 2.0 ** -7)
    assert (d >= lo).all() and (d <= hi).all()


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_golden_generated_blocks_are_the_generator_output(golden, qtype):
    # the fixtures' "gen" blocks are the generator's stream (seed 1234, tensor 7), so the
    # generator itself is pinned as well as the decode
    key = oracle.stream_key(1234, 7)
    pre = oracle.GOLDEN_PREFIX[qtype]
    assert np.array_equal(golden[f"{pre}_gen_blocks"], oracle.fill(qtype, key, 0, 64))
