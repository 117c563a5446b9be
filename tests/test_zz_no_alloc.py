"""kq_matvec_q4k_noalloc: the tensor-core Q4_K matvec for callers that cannot allocate device
memory (graph-capture regions, servers whose pools already hold the GPU, latency-critical paths).
Its scratch is a static device array shared by all calls, so this file runs last (a failure here
leaves every other test already run). Each case runs two calls in a row and checks both against
the oracle (|y - y_ref| <= 1e-3 * sum|w x|) and against the allocating entry point, at every
scratch width (batch padded to 16, 32 and 64) and at the two shapes that fill the 1 MiB scratch
exactly (k = 8192 at batch 40, k = 32768 at batch 16). It passes alone in a fresh process too."""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.mark.parametrize("rows,K,batches", [
    (1500, 4096, (3, 20)),     # npad 16, then 32
    (640, 8192, (40, 40)),     # npad 64: k * 64 * 2 = 1 MiB, the whole scratch
    (300, 32768, (16, 9)),     # npad 16: k * 16 * 2 = 1 MiB
])
def test_noalloc_matches_the_oracle_and_the_allocating_entry_point_twice(kernels, rows, K, batches):
    L = kb.lib()
    n = rows * K // 256
    W = torch.empty(n * 144, dtype=torch.uint8, device="cuda")
    kernels.fill(4, W, 0, n, kb.stream_key(404 + K, 4))
    Wh = W.cpu().numpy()
    for call, batch in enumerate(batches):
        x = np.random.default_rng(call + K).standard_normal((batch, K), dtype=np.float32)
        xd = torch.from_numpy(x).cuda()
        y_new = torch.full((batch, rows), float("nan"), device="cuda")
        y_old = torch.full((batch, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = L.kq_matvec_q4k_noalloc(y_new.data_ptr(), W.data_ptr(), xd.data_ptr(), rows, K, batch, None)
        assert rc == 0, kb.last_error()
        kernels.matvec(4, y_old, W, xd, rows, K, batch, flags=kb.FLAG_TENSOR_CORES)
        torch.cuda.synchronize()
        a, b = y_new.cpu().numpy().astype(np.float64), y_old.cpu().numpy().astype(np.float64)
        y_ref, bound = oracle.matvec_ref(4, Wh, x, K, 0, rows)
        assert np.isfinite(a).all()
        assert (np.abs(a - y_ref) <= TOL * bound).all(), f"call {call}: worst {(np.abs(a - y_ref) / bound).max():.3e}"
        assert (np.abs(a - b) <= TOL * bound).all(), f"call {call} vs the allocating path"
    kernels.device_error()


def test_noalloc_rejects_sizes_past_its_static_scratch(kernels):
    L = kb.lib()
    W = torch.empty(144 * 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(64 * 16384, device="cuda")
    y = torch.zeros(64, device="cuda")
    rc = L.kq_matvec_q4k_noalloc(y.data_ptr(), W.data_ptr(), x.data_ptr(), 1, 16384, 64, None)
    assert rc == kb.KQ_E_INVALID
    assert "static" in kb.last_error()
