"""Parity of the CUDA path with the CPU oracle, through the C ABI (libkq.so).

Bars:
* dequantised weights bit-exact with the oracle decode (itself pinned to gguf-py 0.19.0);
* every output |y - y_ref| <= 1e-3 * sum_k |w_k x_k|   (TOL below), y_ref and the sum in f64.
Shapes follow the reference's testing habit of edge sweeps (examples/matmul/src/tests.rs:41-165):
rows around the SM count and tile sizes, one-block rows, the 43-block K=11008 Q6_K rows that
start off 16-byte boundaries, NaN canaries past the outputs, and integer inputs that are exact
in any summation order (examples/matmul/src/tests.rs:167-171).
"""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

TOL = 1e-3  # |y - y_ref| <= TOL * sum|w x|


def dev_weights(kernels, qtype, rows, K, key):
    n = rows * K // 256
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, n, key)
    return W


def run_matvec(kernels, qtype, W, x, rows, K, **kw):
    batch = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, batch, **kw)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def check(y, y_ref, bound, what=""):
    err = np.abs(y.astype(np.float64) - y_ref)
    ok = err <= TOL * bound
    assert np.isfinite(y).all(), f"{what}: non-finite outputs"
    assert ok.all(), f"{what}: {np.count_nonzero(~ok)} outputs out of tolerance, worst ratio " \
                     f"{(err / np.maximum(bound, 1e-300)).max():.3e}"


# ---------------------------------------------------------------- generator and decode

@pytest.mark.parametrize("qtype", [4, 6])
def test_device_fill_matches_oracle(kernels, qtype):
    key = kb.stream_key(11, qtype)
    b0, n = 123, 4000
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, b0, n, key)
    torch.cuda.synchronize()
    assert np.array_equal(W.cpu().numpy(), oracle.fill(qtype, key, b0, n))


@pytest.mark.parametrize("qtype", [4, 6])
@pytest.mark.parametrize("which", ["gen", "raw", "kat"])
def test_device_dequant_matches_golden(kernels, golden, qtype, which):
    blocks = golden[f"q{qtype}k_{which}_blocks"]
    want = golden[f"q{qtype}k_{which}_f32bits"]
    n = blocks.size // kb.block_bytes(qtype)
    W = torch.from_numpy(blocks.copy()).cuda()
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(qtype, out, W, n)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    nan = np.isnan(want.view(np.float32))
    assert np.array_equal(np.isnan(got.view(np.float32)), nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("qtype", [4, 6])
def test_device_dequant_matches_oracle_on_generated(kernels, qtype):
    n = 20000
    W = dev_weights(kernels, qtype, n, 256, kb.stream_key(3, qtype))
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(qtype, out, W, n)
    torch.cuda.synchronize()
    want = oracle.dequant(qtype, W.cpu().numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


# ---------------------------------------------------------------- matvec parity

SHAPES = [
    # (qtype, rows, K, batch)
    (4, 1, 256, 1), (4, 7, 512, 1), (4, 148, 4096, 1), (4, 149, 4096, 1), (4, 1000, 4096, 1),
    (4, 4096, 4096, 1), (4, 300, 11008, 1), (4, 64, 28672, 1), (4, 257, 8192, 1),
    (6, 1, 256, 1), (6, 7, 512, 1), (6, 147, 4096, 1), (6, 1001, 4096, 1), (6, 333, 11008, 1),
    (6, 64, 28672, 1), (6, 513, 8192, 1), (6, 3, 11008, 1),
    (4, 500, 4096, 2), (4, 300, 4096, 3), (4, 301, 4096, 4), (4, 150, 4096, 5), (4, 200, 4096, 8),
    (6, 500, 4096, 2), (6, 299, 4096, 3), (6, 301, 4096, 4), (6, 151, 4096, 7), (6, 200, 4096, 8),
    (4, 100, 11008, 2), (6, 100, 11008, 2),
    # K-tiled rows with whole 16-row bands (tensor-map tiles on the warp-MMA kernel) and a last
    # band of a few rows; Q6_K at K = 16384 and 28672 takes x in two parts (two bands a CTA here)
    (4, 3000, 8192, 1), (6, 2400, 16384, 1), (4, 2400, 8192, 2), (4, 2600, 12288, 2),
    (6, 4096, 28672, 1),
]


@pytest.mark.parametrize("path", ["auto", "cuda_cores"])
@pytest.mark.parametrize("qtype,rows,K,batch", SHAPES)
def test_matvec_matches_oracle(kernels, qtype, rows, K, batch, path):
    key = kb.stream_key(1000 + rows, K * 10 + qtype)
    W = dev_weights(kernels, qtype, rows, K, key)
    x = np.random.default_rng(rows * 7 + K + batch).standard_normal((batch, K), dtype=np.float32)
    flags = kb.FLAG_CUDA_CORES if path == "cuda_cores" else 0
    y = run_matvec(kernels, qtype, W, x, rows, K, flags=flags)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"q{qtype} {rows}x{K} b{batch}")


@pytest.mark.parametrize("qtype", [4, 6])
def test_matvec_simple_entry_points(kernels, qtype):
    rows, K = 333, 4096
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(5, qtype))
    x = np.random.default_rng(9).standard_normal((2, K), dtype=np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(2 * rows, dtype=torch.float32, device="cuda")
    fn = kernels.matvec_q4k if qtype == 4 else kernels.matvec_q6k
    fn(y, W, xd, rows, K, 2)
    torch.cuda.synchronize()
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y.cpu().numpy().reshape(2, rows), y_ref, bound)


@pytest.mark.parametrize("qtype", [4, 6])
def test_matvec_golden_fixture(kernels, golden, qtype):
    W = torch.from_numpy(golden[f"q{qtype}k_mv_W"].copy()).cuda()
    x = golden[f"q{qtype}k_mv_x"]
    y = run_matvec(kernels, qtype, W, x, 8, 512)
    check(y, golden[f"q{qtype}k_mv_y"], golden[f"q{qtype}k_mv_bound"])


@pytest.mark.parametrize("qtype", [4, 6])
def test_matvec_integer_inputs_are_exact(kernels, qtype):
    # power-of-two scales and small-integer x: every partial sum is exact in f32, in any order
    rows, K, batch = 300, 1024, 3
    Wn = oracle.fill(qtype, oracle.stream_key(77, qtype), 0, rows * K // 256)
    bb = kb.block_bytes(qtype)
    blocks = Wn.reshape(-1, bb)
    if qtype == 4:
        blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
        blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    else:
        blocks[:, 208:210] = np.array([0x1C00], dtype=np.uint16).view(np.uint8)  # d = 2^-8
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(3).integers(-2, 3, size=(batch, K)).astype(np.float32)
    y = run_matvec(kernels, qtype, W, x, rows, K)
    y_ref, _ = oracle.matvec_ref(qtype, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


@pytest.mark.parametrize("qtype", [4, 6])
def test_outputs_do_not_spill_past_the_end(kernels, qtype):
    rows, K, batch = 150, 512, 2
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(8, qtype))
    x = torch.randn(batch, K, device="cuda")
    y = torch.full((batch * rows + 64,), float("nan"), device="cuda")
    kernels.matvec(qtype, y, W, x, rows, K, batch)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    assert np.isfinite(yh[: batch * rows]).all()
    assert np.isnan(yh[batch * rows:]).all()


@pytest.mark.parametrize("qtype", [4, 6])
def test_strided_vectors(kernels, qtype):
    rows, K, batch, ldx, ldy = 200, 1024, 3, 1024 + 36, 200 + 5
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(12, qtype))
    xs = np.random.default_rng(4).standard_normal((batch, ldx), dtype=np.float32)
    xd = torch.from_numpy(xs).cuda()
    y = torch.full((batch, ldy), float("nan"), device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, batch, ldx=ldx, ldy=ldy)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), np.ascontiguousarray(xs[:, :K]), K, 0, rows)
    check(yh[:, :rows], y_ref, bound)
    assert np.isnan(yh[:, rows:]).all()


@pytest.mark.parametrize("qtype", [4, 6])
def test_rmsnorm_prologue(kernels, qtype):
    rows, K, eps = 260, 4096, 1e-6
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(13, qtype))
    x = (np.random.default_rng(6).standard_normal((1, K)) * 3.0).astype(np.float32)
    y = run_matvec(kernels, qtype, W, x, rows, K, prologue=kb.PROLOGUE_RMSNORM, eps=eps)
    xn = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + eps)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), xn.astype(np.float32), K, 0, rows)
    check(y, y_ref, bound)


@pytest.mark.parametrize("qtype", [4, 6])
def test_pair_product_epilogue(kernels, qtype):
    rows, K, scale = 2 * 301, 4096, 0.125
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(14, qtype))
    x = np.random.default_rng(7).standard_normal((1, K), dtype=np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((rows // 2 + 8,), float("nan"), device="cuda")
    kernels.matvec(qtype, y, W, xd, rows, K, 1, epilogue=kb.EPILOGUE_PAIR_PRODUCT, pair_scale=scale)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    r, b = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    v0, v1, b0, b1 = r[0, 0::2], r[0, 1::2], b[0, 0::2], b[0, 1::2]
    want = v0 * v1 * scale
    tol = TOL * (b0 * np.abs(v1) + b1 * np.abs(v0) + TOL * b0 * b1) * scale
    assert (np.abs(yh[: rows // 2] - want) <= tol).all()
    assert np.isnan(yh[rows // 2:]).all()


@pytest.mark.parametrize("qtype,K", [(4, 4096), (6, 4096), (6, 11008)])
@pytest.mark.parametrize("path", ["auto", "cuda_cores"])
def test_silu_product_epilogue(kernels, qtype, K, path):
    # y[r/2] = silu(v(r)) * v(r+1) * scale: a gated FFN's interleaved gate and up rows. silu has
    # slope in [-0.1, 1.1], so the gate's error bound passes through it scaled by at most 1.1.
    rows, scale = 2 * 211, 0.25
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(15, qtype))
    x = np.random.default_rng(8).standard_normal((1, K), dtype=np.float32)
    y = torch.full((rows // 2 + 8,), float("nan"), device="cuda")
    flags = kb.FLAG_CUDA_CORES if path == "cuda_cores" else 0
    kernels.matvec(qtype, y, W, torch.from_numpy(x).cuda(), rows, K, 1,
                   epilogue=kb.EPILOGUE_SILU_PRODUCT, pair_scale=scale, flags=flags)
    torch.cuda.synchronize()
    yh = y.cpu().numpy().astype(np.float64)
    r, b = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    v0, v1, b0, b1 = r[0, 0::2], r[0, 1::2], b[0, 0::2], b[0, 1::2]
    s0 = v0 / (1.0 + np.exp(-v0))
    want = s0 * v1 * scale
    tol = (TOL * (1.1 * b0 * np.abs(v1) + b1 * np.abs(s0) + 1.1 * TOL * b0 * b1) * scale
           + 1e-6 * np.abs(want))
    assert (np.abs(yh[: rows // 2] - want) <= tol).all()
    assert np.isnan(yh[rows // 2:]).all()


def test_invalid_arguments_are_rejected_before_launch(kernels):
    W = torch.empty(144 * 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4096 * 9, device="cuda")
    y = torch.zeros(4096 * 9, device="cuda")
    cases = [
        dict(rows=4, k=300, batch=1),
        dict(rows=4, k=256, batch=0),
        dict(rows=4, k=256, batch=65),
        dict(rows=0, k=256, batch=1),
    ]
    for c in cases:
        with pytest.raises(kb.Error) as e:
            kernels.matvec(4, y, W, x, c["rows"], c["k"], c["batch"])
        assert e.value.code == kb.KQ_E_INVALID
    with pytest.raises(kb.Error) as e:  # misaligned weights
        kernels.matvec(4, y, W.data_ptr() + 2, x, 4, 256, 1)
    assert e.value.code == kb.KQ_E_INVALID
    with pytest.raises(kb.Error) as e:  # odd rows with the pair epilogue
        kernels.matvec(4, y, W, x, 3, 256, 1, epilogue=kb.EPILOGUE_PAIR_PRODUCT)
    assert e.value.code == kb.KQ_E_INVALID
    kernels.device_error()


# ---------------------------------------------------------------- BASELINE.json shapes

@pytest.mark.parametrize("qtype,rows,K", [(4, 4096, 4096), (6, 32000, 4096)])
def test_config_shapes_full_check(kernels, qtype, rows, K):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(2026, qtype))
    x = np.random.default_rng(2026).standard_normal((1, K), dtype=np.float32)
    y = run_matvec(kernels, qtype, W, x, rows, K)
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"config q{qtype} {rows}x{K}")


@pytest.mark.parametrize("batch", [1, 2, 4, 8])
def test_sweep_shape_full_check(kernels, batch):
    rows, K = 14336, 4096
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(2027, 4))
    x = np.random.default_rng(batch).standard_normal((batch, K), dtype=np.float32)
    y = run_matvec(kernels, 4, W, x, rows, K)
    y_ref, bound = oracle.matvec_ref(4, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"sweep b{batch}")


@pytest.mark.parametrize("qtype,rows,K", [(6, 8192, 28672), (4, 28672, 8192)])
def test_70b_shapes_sampled_rows_and_linearity(kernels, qtype, rows, K):
    W = dev_weights(kernels, qtype, rows, K, kb.stream_key(70, qtype))
    rng = np.random.default_rng(70)
    x1 = rng.standard_normal((1, K), dtype=np.float32)
    x2 = rng.standard_normal((1, K), dtype=np.float32)
    y1 = run_matvec(kernels, qtype, W, x1, rows, K)
    y2 = run_matvec(kernels, qtype, W, x2, rows, K)
    y12 = run_matvec(kernels, qtype, W, x1 + x2, rows, K)
    Wh = W.cpu().numpy()
    for r0 in (0, rows // 2 - 17, rows - 40):
        y_ref, bound = oracle.matvec_ref(qtype, Wh, x1, K, r0, r0 + 40)
        check(y1[:, r0:r0 + 40], y_ref, bound)
    # linearity at full size: y(x1 + x2) = y(x1) + y(x2) within the summed bounds
    _, b1 = oracle.matvec_ref(qtype, Wh, np.abs(x1) + np.abs(x2), K, 0, 64)
    assert (np.abs(y12[:, :64] - y1[:, :64] - y2[:, :64]) <= 3 * TOL * b1).all()
    assert np.isfinite(y12).all()


# ---------------------------------------------------------------- tensor-core (tcgen05) path

TC_SHAPES = [
    # (rows, K, batch)
    (1, 256, 1), (100, 256, 1), (128, 512, 1), (129, 4096, 1), (300, 11008, 1), (4096, 4096, 1),
    (333, 4096, 2), (257, 4096, 8), (333, 4096, 17), (77, 8192, 33), (1000, 4096, 64),
    (14336, 4096, 16), (5000, 4096, 40),
    # one- and two-row tiles; several tiles per CTA (rows past 148 x 128); the sweep shape at 32, 64
    (2, 512, 12), (16, 256, 9), (20000, 2048, 16), (40000, 1024, 64), (14336, 4096, 32), (14336, 4096, 64),
]


@pytest.mark.parametrize("rows,K,batch", TC_SHAPES)
def test_tensor_core_matvec_matches_oracle(kernels, rows, K, batch):
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(3000 + rows, K + batch))
    x = np.random.default_rng(rows + K + batch).standard_normal((batch, K), dtype=np.float32)
    y = run_matvec(kernels, 4, W, x, rows, K, flags=kb.FLAG_TENSOR_CORES)
    y_ref, bound = oracle.matvec_ref(4, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"tc {rows}x{K} b{batch}")


def test_tensor_core_integer_inputs_are_exact(kernels):
    rows, K, batch = 300, 1024, 5
    Wn = oracle.fill(4, oracle.stream_key(78, 4), 0, rows * K // 256)
    blocks = Wn.reshape(-1, 144)
    blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
    blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(4).integers(-2, 3, size=(batch, K)).astype(np.float32)
    y = run_matvec(kernels, 4, W, x, rows, K, flags=kb.FLAG_TENSOR_CORES)
    y_ref, _ = oracle.matvec_ref(4, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


def test_tensor_core_strided_and_canaries(kernels):
    rows, K, batch, ldx, ldy = 211, 2048, 19, 2048 + 20, 211 + 13
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(31, 4))
    xs = np.random.default_rng(31).standard_normal((batch, ldx), dtype=np.float32)
    xd = torch.from_numpy(xs).cuda()
    y = torch.full((batch, ldy), float("nan"), device="cuda")
    kernels.matvec(4, y, W, xd, rows, K, batch, ldx=ldx, ldy=ldy, flags=kb.FLAG_TENSOR_CORES)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    y_ref, bound = oracle.matvec_ref(4, W.cpu().numpy(), np.ascontiguousarray(xs[:, :K]), K, 0, rows)
    check(yh[:, :rows], y_ref, bound)
    assert np.isnan(yh[:, rows:]).all()


@pytest.mark.parametrize("batch", [1, 4, 8])
def test_both_paths_agree(kernels, batch):
    rows, K = 1500, 4096
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(32, batch))
    x = np.random.default_rng(batch).standard_normal((batch, K), dtype=np.float32)
    y_tc = run_matvec(kernels, 4, W, x, rows, K, flags=kb.FLAG_TENSOR_CORES)
    y_cc = run_matvec(kernels, 4, W, x, rows, K, flags=kb.FLAG_CUDA_CORES)
    _, bound = oracle.matvec_ref(4, W.cpu().numpy(), x, K, 0, rows)
    assert (np.abs(y_tc - y_cc) <= 2 * TOL * bound).all()


def test_path_flags_are_checked(kernels):
    W = torch.empty(144 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4096 * 64, device="cuda")
    y = torch.zeros(4096 * 64, device="cuda")
    with pytest.raises(kb.Error) as e:
        kernels.matvec(4, y, W, x, 1, 4096, 1, flags=kb.FLAG_TENSOR_CORES | kb.FLAG_CUDA_CORES)
    assert e.value.code == kb.KQ_E_INVALID
    with pytest.raises(kb.Error) as e:  # Q6_K has no tensor-core kernel yet
        kernels.matvec(6, y, W, x, 1, 256, 1, flags=kb.FLAG_TENSOR_CORES)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:  # the CUDA cores stop at batch 8
        kernels.matvec(4, y, W, x, 1, 256, 9, flags=kb.FLAG_CUDA_CORES)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    kernels.device_error()


@pytest.mark.parametrize("mag", [1e-25, 1e-3, 1e19, 1e30])
def test_rmsnorm_prologue_any_magnitude(kernels, mag):
    # the norm's sum of squares must not overflow or underflow for any finite x
    rows, K, eps = 150, 2048, 1e-6
    W = dev_weights(kernels, 4, rows, K, kb.stream_key(15, 4))
    x = (np.random.default_rng(8).standard_normal((1, K)) * mag).astype(np.float32)
    y = run_matvec(kernels, 4, W, x, rows, K, prologue=kb.PROLOGUE_RMSNORM, eps=eps)
    x64 = x.astype(np.float64)
    xn = x64 / np.sqrt(np.mean(x64 ** 2) + eps)
    y_ref, bound = oracle.matvec_ref(4, W.cpu().numpy(), xn.astype(np.float32), K, 0, rows)
    check(y, y_ref, bound, f"rmsnorm x~{mag}")


@pytest.mark.parametrize("qtype,rows,K,batch,pad", [(6, 1000, 4096, 1, 0), (4, 300, 2048, 4, 8),
                                                    (4, 64, 1024, 8, 0), (6, 77, 11008, 1, 4)])
def test_matvec_host_buffers_match_the_device_path(kernels, qtype, rows, K, batch, pad):
    # kq_matvec_host: x and y in host memory (pinned torch and plain numpy), strided, equal bit
    # for bit to the same matvec on device buffers
    W = torch.empty(kb.matrix_bytes(qtype, rows, K), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, rows * K // 256, kb.stream_key(95, qtype))
    ldx, ldy = K + 4 * pad, rows + pad
    x = np.random.default_rng(95).standard_normal((batch, ldx), dtype=np.float32)
    yd = torch.zeros((batch, ldy), dtype=torch.float32, device="cuda")
    kernels.matvec(qtype, yd, W, torch.from_numpy(x).cuda(), rows, K, batch, ldx=ldx, ldy=ldy)
    torch.cuda.synchronize()
    want = yd.cpu().numpy()
    for pinned in (True, False):
        if pinned:
            xh = torch.from_numpy(x).pin_memory()
            yh = torch.full((batch, ldy), -7.0, dtype=torch.float32).pin_memory()
        else:
            xh = x.copy()
            yh = np.full((batch, ldy), -7.0, dtype=np.float32)
        kernels.matvec_host(qtype, yh, W, xh, rows, K, batch, ldx=ldx, ldy=ldy)
        torch.cuda.synchronize()
        got = yh.numpy() if pinned else yh
        assert np.array_equal(got[:, :rows], want[:, :rows])
        assert (got[:, rows:] == -7.0).all()  # the gaps between rows of y stay untouched


def test_matvec_host_rejects_device_arrays(kernels):
    W = torch.empty(kb.matrix_bytes(4, 16, 256), dtype=torch.uint8, device="cuda")
    with pytest.raises(kb.Error):
        kernels.matvec_host(4, torch.zeros(16, device="cuda"), W, np.zeros(256, np.float32), 16, 256)
