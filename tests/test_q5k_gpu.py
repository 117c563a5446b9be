"""Q5_K on the GPU, through the C ABI: the device generator and decoder bit for bit against the
CPU oracle and the gguf-py fixtures, and the matvec (the warp-MMA kernel's integer path at batch 1,
the tensor-core kernel at batch 2..64) against the oracle's f64 reference.

Q5_K is Q4_K's block (f16 d and dmin, twelve bytes of 6-bit sub-block scales and mins, 128 bytes of
nibbles) with 32 more bytes, qh, whose bit g of byte l is the fifth bit of element 32 g + l
(gguf-py/gguf/quants.py Q5_K.dequantize_blocks). The shapes sweep the kernel's seams as for Q4_K:
partial bands of 16 rows, the fixed-block loop (whole-row tiles on 16-byte boundaries), the
turns loop (K = 11008 rows 16 mod 128 bytes, K-tiled rows), and split tiles (K = 4096: 2816-byte
rows, 0 mod 128). Bar: |y - y_ref| <= 1e-3 * sum_k |w_k x_k| per output.
"""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

TOL = 1e-3
OTHER_WARPS = 1 << 29  # the other consumer-warp arrangement (turns <-> one warp per block)


def dev_weights(kernels, rows, K, key):
    n = rows * K // 256
    W = torch.empty(n * kb.Q5K_BYTES, dtype=torch.uint8, device="cuda")
    kernels.fill(5, W, 0, n, key)
    return W


def run(kernels, W, x, rows, K, **kw):
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.full((x.shape[0], rows), float("nan"), dtype=torch.float32, device="cuda")
    kernels.matvec(5, y, W, xd, rows, K, x.shape[0], **kw)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def check(y, y_ref, bound, what=""):
    err = np.abs(y.astype(np.float64) - y_ref)
    assert np.isfinite(y).all(), f"{what}: non-finite outputs"
    assert (err <= TOL * bound).all(), \
        f"{what}: worst ratio {(err / np.maximum(bound, 1e-300)).max():.3e}"


def test_q5k_device_fill_matches_oracle(kernels):
    key = kb.stream_key(11, 5)
    b0, n = 123, 4000
    W = torch.empty(n * kb.Q5K_BYTES, dtype=torch.uint8, device="cuda")
    kernels.fill(5, W, b0, n, key)
    torch.cuda.synchronize()
    assert np.array_equal(W.cpu().numpy(), oracle.fill(5, key, b0, n))


@pytest.mark.parametrize("which", ["gen", "raw", "kat"])
def test_q5k_device_dequant_matches_golden(kernels, golden, which):
    blocks = golden[f"q5k_{which}_blocks"]
    want = golden[f"q5k_{which}_f32bits"]
    n = blocks.size // kb.Q5K_BYTES
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(5, out, torch.from_numpy(blocks.copy()).cuda(), n)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    nan = np.isnan(want.view(np.float32))
    assert np.array_equal(np.isnan(got.view(np.float32)), nan)
    assert np.array_equal(got[~nan], want[~nan])


def test_q5k_device_dequant_matches_oracle_on_generated(kernels):
    n = 20000
    W = dev_weights(kernels, n, 256, kb.stream_key(3, 5))
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(5, out, W, n)
    torch.cuda.synchronize()
    want = oracle.dequant(5, W.cpu().numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


SHAPES = [  # (rows, K)
    (1, 256), (15, 256), (16, 512), (17, 4096), (148, 4096), (300, 4096), (4096, 4096),
    (1000, 4352), (257, 8192), (300, 11008), (3, 11008), (64, 28672), (77, 2816),
    # K-tiled rows with whole 16-row bands (tensor-map tiles) and a last band of a few rows
    (4096, 8192), (2500, 16384),
]


@pytest.mark.parametrize("rows,K", SHAPES)
@pytest.mark.parametrize("arrangement", [0, OTHER_WARPS])
def test_q5k_matvec_matches_oracle(kernels, rows, K, arrangement):
    W = dev_weights(kernels, rows, K, kb.stream_key(6000 + rows, K))
    x = np.random.default_rng(rows + K).standard_normal((1, K), dtype=np.float32)
    y = run(kernels, W, x, rows, K, flags=arrangement)
    y_ref, bound = oracle.matvec_ref(5, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"q5 {rows}x{K} arrangement {arrangement}")


def test_q5k_matvec_golden_fixture(kernels, golden):
    W = torch.from_numpy(golden["q5k_mv_W"].copy()).cuda()
    x = golden["q5k_mv_x"]
    for b in range(x.shape[0]):  # batch 1, one vector at a time
        y = run(kernels, W, x[b:b + 1], 8, 512)
        check(y, golden["q5k_mv_y"][b:b + 1], golden["q5k_mv_bound"][b:b + 1], f"vector {b}")


def test_q5k_matvec_integer_inputs_are_exact(kernels):
    # power-of-two d and dmin, small-integer x: every product and partial sum is exact
    rows, K = 300, 1024
    blocks = oracle.fill(5, oracle.stream_key(79, 5), 0, rows * K // 256).reshape(-1, kb.Q5K_BYTES)
    blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
    blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(5).integers(-2, 3, size=(1, K)).astype(np.float32)
    y = run(kernels, W, x, rows, K)
    y_ref, _ = oracle.matvec_ref(5, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


def test_q5k_matvec_every_fifth_bit_counts(kernels):
    # qh all ones versus all zeros moves each output by exactly 16 * d * scale * sum(x) per
    # sub-block: compare both against the oracle, and check they differ
    rows, K = 64, 2048
    base = oracle.fill(5, oracle.stream_key(90, 5), 0, rows * K // 256).reshape(-1, kb.Q5K_BYTES)
    x = np.random.default_rng(90).standard_normal((1, K), dtype=np.float32)
    ys = []
    for fill in (0x00, 0xFF):
        blocks = base.copy()
        blocks[:, 16:48] = fill
        W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
        y = run(kernels, W, x, rows, K)
        y_ref, bound = oracle.matvec_ref(5, blocks.reshape(-1), x, K, 0, rows)
        check(y, y_ref, bound, f"qh {fill:#x}")
        ys.append(y)
    assert not np.array_equal(ys[0], ys[1])


@pytest.mark.parametrize("mag", [1e-30, 1.0, 1e30])
def test_q5k_matvec_any_magnitude_and_rmsnorm(kernels, mag):
    rows, K, eps = 150, 4096, 1e-6
    W = dev_weights(kernels, rows, K, kb.stream_key(82, 5))
    x = (np.random.default_rng(82).standard_normal((1, K)) * mag).astype(np.float32)
    y = run(kernels, W, x, rows, K)
    y_ref, bound = oracle.matvec_ref(5, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"x~{mag}")
    y = run(kernels, W, x, rows, K, prologue=kb.PROLOGUE_RMSNORM, eps=eps)
    x64 = x.astype(np.float64)
    xn = (x64 / np.sqrt(np.mean(x64 ** 2) + eps)).astype(np.float32)
    y_ref, bound = oracle.matvec_ref(5, W.cpu().numpy(), xn, K, 0, rows)
    check(y, y_ref, bound, f"rmsnorm x~{mag}")


def test_q5k_matvec_is_deterministic(kernels):
    rows, K = 2000, 4096
    W = dev_weights(kernels, rows, K, kb.stream_key(80, 5))
    x = np.random.default_rng(80).standard_normal((1, K), dtype=np.float32)
    y1 = run(kernels, W, x, rows, K)
    y2 = run(kernels, W, x, rows, K)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


def test_q5k_matvec_rejects_what_it_does_not_serve(kernels):
    W = torch.zeros(kb.Q5K_BYTES * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4096 * 65, device="cuda")
    y = torch.zeros(4096 * 65, device="cuda")
    with pytest.raises(kb.Error) as e:  # the CUDA-core kernel does not take Q5_K
        kernels.matvec(5, y, W, x, 1, 256, 1, flags=kb.FLAG_CUDA_CORES)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:  # the warp-MMA kernel serves Q5_K at batch 1 only
        kernels.matvec(5, y, W, x, 1, 256, 2, flags=kb.FLAG_WARP_MMA)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:  # no fused prologue above batch 1
        kernels.matvec(5, y, W, x, 1, 256, 2, prologue=kb.PROLOGUE_RMSNORM, eps=1e-6)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error):  # batch 65
        kernels.matvec(5, y, W, x, 1, 256, 65)


# ---------------------------------------------------------------- batch 2..64: the tensor-core kernel

TC_SHAPES = [  # (rows, K, batch)
    (1, 256, 2), (16, 512, 9), (100, 4096, 16), (300, 11008, 3), (333, 4096, 17), (77, 2816, 33),
    (1000, 4096, 64), (14336, 4096, 16), (5000, 4352, 40), (20000, 2048, 24),
]


@pytest.mark.parametrize("rows,K,batch", TC_SHAPES)
def test_q5k_tensor_core_matmul_matches_oracle(kernels, rows, K, batch):
    W = dev_weights(kernels, rows, K, kb.stream_key(7000 + rows, K + batch))
    x = np.random.default_rng(rows + K + batch).standard_normal((batch, K), dtype=np.float32)
    y = run(kernels, W, x, rows, K)
    y_ref, bound = oracle.matvec_ref(5, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, f"q5 tc {rows}x{K} b{batch}")


def test_q5k_tensor_core_every_fifth_bit_counts(kernels):
    rows, K, batch = 200, 2048, 12
    base = oracle.fill(5, oracle.stream_key(91, 5), 0, rows * K // 256).reshape(-1, kb.Q5K_BYTES)
    x = np.random.default_rng(91).standard_normal((batch, K), dtype=np.float32)
    ys = []
    for fill in (0x00, 0xFF, 0x5A):
        blocks = base.copy()
        blocks[:, 16:48] = fill
        W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
        y = run(kernels, W, x, rows, K)
        y_ref, bound = oracle.matvec_ref(5, blocks.reshape(-1), x, K, 0, rows)
        check(y, y_ref, bound, f"qh {fill:#x}")
        ys.append(y)
    assert not np.array_equal(ys[0], ys[1]) and not np.array_equal(ys[1], ys[2])


def test_q5k_tensor_core_integer_inputs_are_exact(kernels):
    rows, K, batch = 300, 1024, 5
    blocks = oracle.fill(5, oracle.stream_key(92, 5), 0, rows * K // 256).reshape(-1, kb.Q5K_BYTES)
    blocks[:, 0:2] = np.array([0x2400], dtype=np.uint16).view(np.uint8)  # d = 2^-6
    blocks[:, 2:4] = np.array([0x2800], dtype=np.uint16).view(np.uint8)  # dmin = 2^-5
    W = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    x = np.random.default_rng(6).integers(-2, 3, size=(batch, K)).astype(np.float32)
    y = run(kernels, W, x, rows, K)
    y_ref, _ = oracle.matvec_ref(5, blocks.reshape(-1), x, K, 0, rows)
    assert np.array_equal(y, y_ref.astype(np.float32))


def test_q5k_batch_one_on_the_tensor_cores_when_asked(kernels):
    rows, K = 700, 4096
    W = dev_weights(kernels, rows, K, kb.stream_key(93, 5))
    x = np.random.default_rng(93).standard_normal((1, K), dtype=np.float32)
    y = run(kernels, W, x, rows, K, flags=kb.FLAG_TENSOR_CORES)
    y_ref, bound = oracle.matvec_ref(5, W.cpu().numpy(), x, K, 0, rows)
    check(y, y_ref, bound, "q5 tc batch 1")
