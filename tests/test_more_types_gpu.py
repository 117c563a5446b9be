"""Q2_K, Q3_K and Q8_0 on the GPU, through the C ABI: the device decoder bit for bit against the
gguf-py fixtures and the CPU oracle. The library does not multiply these types
yet; kq_matvec refuses them. The kernels run the __host__ __device__ functions of
kernite_b200/csrc/kq_decode.cuh, whose host build tests/test_decode_host.py checks on the CPU."""
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


@pytest.mark.parametrize("qtype", [kb.TYPE_Q2_K, kb.TYPE_Q3_K, kb.TYPE_Q8_0])
def test_matvec_refuses_types_it_does_not_multiply(kernels, qtype):
    W = torch.zeros(272 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, device="cuda")
    y = torch.zeros(16, device="cuda")
    with pytest.raises(kb.Error) as e:
        kernels.matvec(qtype, y, W, x, 1, 256, 1)
    assert e.value.code == kb.KQ_E_INVALID
