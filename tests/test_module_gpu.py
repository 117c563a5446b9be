"""The module image path on the GPU: the library's warp-MMA cubin (kq_module_image) loaded with the
CUDA driver API (cuModuleLoadData) in the primary context, as kernite-cuda loads a module, and the
function kq_matvec_plan names launched with cuLaunchKernel, as kernite's launchers do. Its output
equals kq_matvec's bit for bit and the oracle's within 1e-3 * sum|w x|."""
import ctypes

import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8


@pytest.fixture(scope="module")
def image_module():
    cu = ctypes.CDLL("libcuda.so.1")
    torch.cuda.init()
    torch.zeros(1, device="cuda")  # the primary context is current on this thread
    img = kb.module_image()
    buf = ctypes.create_string_buffer(img, len(img))
    mod = ctypes.c_void_p()
    assert cu.cuModuleLoadData(ctypes.byref(mod), buf) == 0
    yield cu, mod
    cu.cuModuleUnload(mod)


@pytest.mark.parametrize("qtype,rows,k,batch,pair", [(6, 32000, 4096, 1, False), (4, 4096, 4096, 1, False),
                                                     (4, 2048, 8192, 1, True), (4, 1500, 4096, 4, False),
                                                     (6, 300, 11008, 1, False), (5, 1024, 4096, 1, False)])
def test_planned_launch_from_the_image_equals_kq_matvec(kernels, image_module, qtype, rows, k, batch, pair):
    cu, mod = image_module
    n = rows * k // 256
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, n, kb.stream_key(66, rows))
    xh = np.random.default_rng(rows).standard_normal((batch, k)).astype(np.float32)
    x = torch.from_numpy(xh).cuda()
    outs = rows // 2 if pair else rows
    kw = dict(epilogue=kb.EPILOGUE_PAIR_PRODUCT if pair else kb.EPILOGUE_NONE, pair_scale=0.05)
    y0 = torch.full((batch, outs), float("nan"), device="cuda")
    y1 = torch.full((batch, outs), float("nan"), device="cuda")
    kernels.matvec(qtype, y0, W, x, rows, k, batch, **kw)
    plan = kernels.matvec_plan(qtype, y1, W, x, rows, k, batch, **kw)
    fn = ctypes.c_void_p()
    assert cu.cuModuleGetFunction(ctypes.byref(fn), mod, plan.kernel) == 0, plan.kernel
    assert cu.cuFuncSetAttribute(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, plan.shared_bytes) == 0
    params = (ctypes.c_void_p * 1)(ctypes.addressof(plan.params))
    torch.cuda.synchronize()
    rc = cu.cuLaunchKernel(fn, plan.grid[0], plan.grid[1], plan.grid[2], plan.block[0], plan.block[1],
                           plan.block[2], plan.shared_bytes, None, params, None)
    assert rc == 0
    assert cu.cuCtxSynchronize() == 0
    kernels.device_error()
    assert torch.equal(y0, y1)
    if not pair:
        ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), xh, k, 0, rows)
        assert (np.abs(y1.cpu().numpy() - ref) <= 1e-3 * bound).all()


def test_plan_refuses_what_the_warp_mma_kernel_does_not_serve(kernels):
    W = torch.zeros(144 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16 * 4096, device="cuda")
    y = torch.zeros(16 * 16, device="cuda")
    with pytest.raises(kb.Error) as e:
        kernels.matvec_plan(4, y, W, x, 16, 256, 16)
    assert e.value.code == kb.KQ_E_UNSUPPORTED
