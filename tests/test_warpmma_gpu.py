"""Parity of the warp-MMA kernel (KQ_FLAG_WARP_MMA: Q4_K batch 1..8, Q6_K batch 1) with the CPU
oracle, through the C ABI.

The kernel splits each row into tiles of up to 16 super-blocks (one warp each) and 16 rows (the
MMA's M), converts x into three signed byte limbs (batch 1: integer MMAs, the default) or f16
hi + lo operands (batch 2..8, and batch 1 with the ALT_BATCH1 bit; hi only for Q6_K and for
tables too large for shared memory) and sums partial rows across warps. The shapes below sweep those seams: rows that
leave a partial band of 16, K that takes one, two, three or seven K-tiles (including the 43-block
K = 11008 rows that start off 16-byte boundaries), every batch size and each x-table mode. The
bar is the north star's: |y - y_ref| <= 1e-3 * sum_k |w_k x_k| per output, y_ref in f64; inputs
that are exact in any summation order must come out bit for bit (the reference's tensor-core test
habit, examples/matmul/src/tests.rs:167-171).
"""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

TOL = 1e-3
WM = kb.FLAG_WARP_MMA


def dev_weights(kernels, qtype, rows, K, key):
    n = rows * K // 256
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, n, key)
    return W


def run(kernels, qtype, W, x, rows, K, **kw):
    batch = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, batch, **kw)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def check(y, y_ref, bound, what=""):
    err = np.abs(y.astype(np.float64) - y_ref)
    assert np.isfinite(y).all(), f"{what}: non-finite outputs"
    ratio = err / np.maximum(bound, 1e-300)
    assert (err <= TOL * bound).all(), f"{what}: worst ratio {ratio.max():.3e}"
    return ratio.max()


SHAPES = [
    # (qtype, rows, K, batch)
    (4, 1, 256, 1), (4, 15, 256, 1), (4, 16, 512, 1), (4, 17, 4096, 1), (4, 148, 4096, 1),
    (4, 300, 4096, 1), (4, 4096, 4096, 1), (4, 1000, 4352, 1), (4, 257, 8192, 1),
    (4, 300, 11008, 1), (4, 64, 28672, 1),
    (4, 500, 4096, 2), (4, 301, 4096, 3), (4, 333, 4096, 4), (4, 150, 4096, 5), (4, 200, 4096, 7),
    (4, 211, 4096, 8), (4, 100, 11008, 2), (4, 90, 11008, 4), (4, 40, 28672, 2), (4, 33, 8192, 8),
    (6, 1, 256, 1), (6, 15, 512, 1), (6, 147, 4096, 1), (6, 1001, 4096, 1), (6, 333, 11008, 1),
    (6, 3, 11008, 1), (6, 64, 28672, 1), (6, 513, 8192, 1), (6, 77, 2816, 1),
]


@pytest.mark.parametrize("qtype,rows,K,batch", SHAPES)
def test_warpmma_matches_oracle(kernels, qtype, rows, K, batch):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(5000 + rows, K * 10 + qtype))
    x = np.random.default_rng(rows + K + batch).standard_normal((batch, K), dtype=np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"wm q{qtype} {rows}x{K} b{batch}")


@pytest.mark.parametrize("qtype,batch", [(4, 1), (4, 3), (4, 8), (6, 1)])
def test_warpmma_integer_inputs_are_exact(kernels, qtype, batch):
    # power-of-two d, small-integer x: every product and partial sum is exact, in any order
    rows, K = 300, 1024
    Wn = oracle.fill(qtype, oracle.stream_key(79, qtype), 0, rows * K // 256)
    blocks = Wn.reshape(-1, kb.block_bytes(qtype))
    if qtype == 4:
        blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
        blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    else:
        blocks[:, 208:210] = np.array([0x1C00], dtype=np.uint16).view(np.uint8)  # d = 2^-8
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(5).integers(-2, 3, size=(batch, K)).astype(np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM)
    y_ref, _ = oracle.matvec_ref(qtype, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


@pytest.mark.parametrize("qtype", [4, 6])
def test_warpmma_is_deterministic(kernels, qtype):
    rows, K = 2000, 4096
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(80, qtype))
    x = np.random.default_rng(80).standard_normal((1, K), dtype=np.float32)
    y1 = run(kernels, qtype, W, x, rows, K, flags=WM)
    y2 = run(kernels, qtype, W, x, rows, K, flags=WM)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


@pytest.mark.parametrize("qtype,batch", [(4, 1), (4, 3), (4, 6), (6, 1)])
def test_warpmma_strided_vectors_and_canaries(kernels, qtype, batch):
    rows, K, ldx, ldy = 203, 2048, 2048 + 36, 203 + 9
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(81, qtype))
    xs = np.random.default_rng(81).standard_normal((batch, ldx), dtype=np.float32)
    xd = torch.from_numpy(xs).cuda()
    y = torch.full((batch, ldy), float("nan"), device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, batch, ldx=ldx, ldy=ldy, flags=WM)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), np.ascontiguousarray(xs[:, :K]), K, 0, rows)
    check(yh[:, :rows], y_ref, bound)
    assert np.isnan(yh[:, rows:]).all()


@pytest.mark.parametrize("qtype", [4, 6])
@pytest.mark.parametrize("mag", [1e-30, 1e-3, 1.0, 3e3, 1e30])
def test_warpmma_any_magnitude(kernels, qtype, mag):
    # x is scaled by a power of two into f16's range and back: tiny and huge x both hold the bar
    rows, K = 150, 2048
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(82, qtype))
    x = (np.random.default_rng(82).standard_normal((1, K)) * mag).astype(np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"x~{mag}")


@pytest.mark.parametrize("qtype", [4, 6])
@pytest.mark.parametrize("mag", [1e-25, 1.0, 1e30])
def test_warpmma_rmsnorm_prologue(kernels, qtype, mag):
    rows, K, eps = 260, 4096, 1e-6
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(83, qtype))
    x = (np.random.default_rng(83).standard_normal((1, K)) * mag).astype(np.float32)
    y = run(kernels, qtype, W, x, rows, K, prologue=kb.PROLOGUE_RMSNORM, eps=eps, flags=WM)
    x64 = x.astype(np.float64)
    xn = x64 / np.sqrt(np.mean(x64 ** 2) + eps)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), xn.astype(np.float32), K, 0, rows)
    check(y, y_ref, bound)


@pytest.mark.parametrize("qtype,K", [(4, 4096), (6, 4096), (4, 11008)])
def test_warpmma_pair_product_epilogue(kernels, qtype, K):
    rows, scale = 2 * 301, 0.125
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(84, qtype))
    x = np.random.default_rng(84).standard_normal((1, K), dtype=np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((rows // 2 + 8,), float("nan"), device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, 1, epilogue=kb.EPILOGUE_PAIR_PRODUCT,
                   pair_scale=scale, flags=WM)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    r, b = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    v0, v1, b0, b1 = r[0, 0::2], r[0, 1::2], b[0, 0::2], b[0, 1::2]
    want = v0 * v1 * scale
    tol = TOL * (b0 * np.abs(v1) + b1 * np.abs(v0) + TOL * b0 * b1) * scale
    assert (np.abs(yh[: rows // 2] - want) <= tol).all()
    assert np.isnan(yh[rows // 2:]).all()


@pytest.mark.parametrize("qtype,rows,K", [(4, 4096, 4096), (6, 32000, 4096)])
def test_warpmma_config_shapes_full_check(kernels, qtype, rows, K):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(2026, qtype))
    x = np.random.default_rng(2026).standard_normal((1, K), dtype=np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"config q{qtype}")


@pytest.mark.parametrize("batch", [1, 2, 4, 8])
def test_warpmma_sweep_shape_full_check(kernels, batch):
    rows, K = 14336, 4096
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(2027, 4))
    x = np.random.default_rng(batch).standard_normal((batch, K), dtype=np.float32)
    y = run(kernels, 4, W, x, rows, K, flags=WM)
    y_ref, bound = oracle.matvec_ref(4, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"sweep b{batch}")


@pytest.mark.parametrize("qtype,batch", [(4, 1), (4, 5), (6, 1)])
def test_warpmma_agrees_with_cuda_cores(kernels, qtype, batch):
    rows, K = 1500, 4096
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(85, batch))
    x = np.random.default_rng(85).standard_normal((batch, K), dtype=np.float32)
    y_wm = run(kernels, qtype, W, x, rows, K, flags=WM)
    y_cc = run(kernels, qtype, W, x, rows, K, flags=kb.FLAG_CUDA_CORES)
    _, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    assert (np.abs(y_wm - y_cc) <= 2 * TOL * bound).all()


def test_warpmma_rejects_what_it_does_not_serve(kernels):
    W = torch.empty(210 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4096 * 16, device="cuda")
    y = torch.zeros(4096 * 16, device="cuda")
    with pytest.raises(kb.Error) as e:  # Q6_K serves batch 1 only
        kernels.matvec(6, y, W, x, 1, 256, 2, flags=WM)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:  # batch above 8
        kernels.matvec(4, y, W, x, 1, 256, 9, flags=WM)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:  # two path flags
        kernels.matvec(4, y, W, x, 1, 256, 1, flags=WM | kb.FLAG_CUDA_CORES)
    assert e.value.code == kb.KQ_E_INVALID
    kernels.device_error()


# A descriptor flag bit the library keeps for itself (not part of include/kq.h): batch 1 on the
# other warp-MMA variant (Q4_K: integer operands instead of f16; Q6_K: f16 instead of integer),
# so both stay covered.
ALT_BATCH1 = 1 << 30


@pytest.mark.parametrize("qtype,rows,K", [(4, 300, 4096), (6, 333, 4096), (6, 77, 11008),
                                          (4, 64, 28672), (6, 40, 28672)])
def test_warpmma_other_batch1_variant_matches_oracle(kernels, qtype, rows, K):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(86, qtype))
    x = np.random.default_rng(86).standard_normal((1, K), dtype=np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM | ALT_BATCH1)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"other batch-1 variant q{qtype} {rows}x{K}")


@pytest.mark.parametrize("qtype", [4, 6])
@pytest.mark.parametrize("variant", [0, ALT_BATCH1])
def test_warpmma_zero_weights_give_exact_zero(kernels, qtype, variant):
    # every weight zero with nonzero scales around it: Q4_K sc = m = 0; Q6_K q = 32 (ql 0,
    # qh bits 2 in every group) -- the sum must be exactly 0, as the reference's dot product is
    rows, K = 100, 2048
    Wn = oracle.fill(qtype, oracle.stream_key(87, qtype), 0, rows * K // 256)
    blocks = Wn.reshape(-1, kb.block_bytes(qtype))
    if qtype == 4:
        blocks[:, 4:16] = 0
    else:
        blocks[:, 0:128] = 0
        blocks[:, 128:192] = 0xAA
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(87).standard_normal((1, K), dtype=np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM | variant)
    assert np.array_equal(y, np.zeros_like(y))


@pytest.mark.parametrize("qtype", [4, 6])
def test_warpmma_other_batch1_variant_integer_inputs_are_exact(kernels, qtype):
    rows, K = 300, 1024
    Wn = oracle.fill(qtype, oracle.stream_key(88, qtype), 0, rows * K // 256)
    blocks = Wn.reshape(-1, kb.block_bytes(qtype))
    if qtype == 4:
        blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
        blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    else:
        blocks[:, 208:210] = np.array([0x1C00], dtype=np.uint16).view(np.uint8)  # d = 2^-8
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(6).integers(-2, 3, size=(1, K)).astype(np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM | ALT_BATCH1)
    y_ref, _ = oracle.matvec_ref(qtype, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


OTHER_WARPS = 1 << 29  # the other consumer-warp arrangement (turns <-> one warp per block)


@pytest.mark.parametrize("qtype,rows,K,batch", [(4, 300, 4096, 1), (4, 130, 4096, 4),
                                                (4, 97, 8192, 8), (6, 333, 4096, 1),
                                                (6, 77, 11008, 1), (4, 50, 28672, 2),
                                                (6, 40, 2048, 1)])
def test_warpmma_other_warp_arrangement_matches_oracle(kernels, qtype, rows, K, batch):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(89, qtype))
    x = np.random.default_rng(89).standard_normal((batch, K), dtype=np.float32)
    y = run(kernels, qtype, W, x, rows, K, flags=WM | OTHER_WARPS)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"other warp arrangement q{qtype} {rows}x{K} b{batch}")
