"""Q2_K, Q3_K and Q8_0 on the GPU, through the C ABI: the device decoder bit for bit against the
gguf-py fixtures and the CPU oracle (the kernels run the __host__ __device__ functions of
kernite_b200/csrc/kq_decode.cuh, whose host build tests/test_decode_host.py checks on the CPU), and
the batch-1 matvec (CUDA-core kernel, kq_types.cu) within 1e-3 * sum|w x| of the oracle and of
the gguf-py fixture matvec."""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

TYPES = [2, 3, 8]


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("which", ["gen", "raw", "kat"])
def test_device_dequant_matches_gguf(kernels, golden, qtype, which):
    pre = oracle.GOLDEN_PREFIX[qtype]
    blocks = golden[f"{pre}_{which}_blocks"]
    want = golden[f"{pre}_{which}_f32bits"]
    n = blocks.size // kb.block_bytes(qtype)
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(qtype, out, torch.from_numpy(blocks.copy()).cuda(), n)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    nan = np.isnan(want.view(np.float32))
    assert np.array_equal(np.isnan(got.view(np.float32)), nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("qtype", TYPES)
def test_device_dequant_matches_oracle_on_generated(kernels, qtype):
    n = 3000
    Wh = oracle.fill(qtype, oracle.stream_key(12, qtype), 77, n)
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    kernels.dequant(qtype, out, torch.from_numpy(Wh).cuda(), n)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), oracle.dequant(qtype, Wh).view(np.uint32))


SHAPES = [(1, 256), (33, 4096), (1000, 4096), (300, 11008), (64, 28672), (4096, 4096)]


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("rows,k", SHAPES)
def test_matvec_matches_oracle(kernels, qtype, rows, k):
    """y within 1e-3 * sum|w x| of the oracle's f64 matvec, odd unit counts per row included
    (K = 11008: 43 units, so Q3_K rows start 2-byte aligned), NaN canaries past y untouched."""
    Wh = oracle.fill(qtype, oracle.stream_key(31, qtype * 1000 + rows), 0, rows * k // 256)
    xh = np.random.default_rng(rows + k).standard_normal(k).astype(np.float32)
    y = torch.full((rows + 8,), float("nan"), device="cuda")
    kernels.matvec(qtype, y, torch.from_numpy(Wh).cuda(), torch.from_numpy(xh).cuda(), rows, k, 1)
    torch.cuda.synchronize()
    kernels.device_error()
    ref, bound = oracle.matvec_ref(qtype, Wh, xh[None, :], k, 0, rows)
    got = y.cpu().numpy()
    assert np.isnan(got[rows:]).all()
    assert (np.abs(got[:rows].astype(np.float64) - ref[0]) <= 1e-3 * bound[0]).all()


@pytest.mark.parametrize("qtype", TYPES)
def test_matvec_matches_gguf_fixture(kernels, golden, qtype):
    """The committed small matvec computed from gguf-py's dequantisation (tests/golden)."""
    pre = oracle.GOLDEN_PREFIX[qtype]
    W, x = golden[f"{pre}_mv_W"], golden[f"{pre}_mv_x"].astype(np.float32)
    want, bound = golden[f"{pre}_mv_y"], golden[f"{pre}_mv_bound"]
    rows, k = want.shape[-1], x.shape[-1]
    Wd = torch.from_numpy(W.copy()).cuda()
    for b in range(x.shape[0]):  # the fixture's vectors one at a time (batch 1)
        y = torch.zeros(rows, device="cuda")
        kernels.matvec(qtype, y, Wd, torch.from_numpy(x[b].copy()).cuda(), rows, k, 1)
        torch.cuda.synchronize()
        assert (np.abs(y.cpu().numpy() - want[b]) <= 1e-3 * bound[b]).all(), b


def test_integer_exact_inputs_give_exact_outputs(kernels):
    """Q8_0 with d = 1 and integer x: every product and sum is an exact small integer."""
    rows, k = 40, 512
    Wh = oracle.fill(8, oracle.stream_key(5, 8), 0, rows * k // 256).reshape(-1, 34)
    Wh[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), dtype=np.uint8)
    Wh = Wh.reshape(-1)
    xh = np.random.default_rng(2).integers(-3, 4, k).astype(np.float32)
    y = torch.zeros(rows, device="cuda")
    kernels.matvec(8, y, torch.from_numpy(Wh).cuda(), torch.from_numpy(xh).cuda(), rows, k, 1)
    torch.cuda.synchronize()
    ref, _ = oracle.matvec_ref(8, Wh, xh[None, :], k, 0, rows)
    assert np.array_equal(y.cpu().numpy().astype(np.float64), ref[0])


@pytest.mark.parametrize("qtype", [kb.TYPE_Q2_K, kb.TYPE_Q3_K, kb.TYPE_Q8_0])
def test_matvec_refuses_what_it_does_not_serve(kernels, qtype):
    W = torch.zeros(272 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(2 * 256, device="cuda")
    y = torch.zeros(32, device="cuda")
    with pytest.raises(kb.Error) as e:
        kernels.matvec(qtype, y, W, x, 1, 256, 2)  # batch 2
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:
        kernels.matvec(qtype, y, W, x, 2, 256, 1, epilogue=kb.EPILOGUE_PAIR_PRODUCT)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
    with pytest.raises(kb.Error) as e:
        kernels.matvec(qtype, y, W, x, 1, 100, 1)  # k not a multiple of 256
    assert e.value.code == kb.KQ_E_INVALID
