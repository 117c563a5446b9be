"""Chains (kq_matvec_chain) on the GPU: several batch-1 matvecs in one launch of the warp-MMA
integer kernel, ordered by counters instead of kernel boundaries. Each chain job's outputs equal
the lone launch's bit for bit (the same consumer code over the same tiles), stacks run as
chains equal the stacks run one launch per projection and the unsharded CPU reference, over
several tokens replayed from a CUDA graph (the step counter keeps advancing), and a wait that can
never be met gives up with the device error word set instead of hanging."""
import dataclasses
import math

import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb
from kernite_b200 import stack as st

pytestmark = pytest.mark.gpu


def _job(qtype, y, w, x, rows, k, counter=0, wait=0, target=0, rmsnorm=False, pair_scale=None):
    j = kb.KqChainJob()
    j.mv = kb.KqMatvecDesc(type={4: kb.TYPE_Q4_K, 5: kb.TYPE_Q5_K, 6: kb.TYPE_Q6_K}[qtype], rows=rows,
                           k=k, batch=1, y=y.data_ptr(), w=w.data_ptr(), x=x.data_ptr(),
                           prologue=kb.PROLOGUE_RMSNORM if rmsnorm else kb.PROLOGUE_NONE,
                           epilogue=kb.EPILOGUE_PAIR_PRODUCT if pair_scale else kb.EPILOGUE_NONE,
                           eps=1e-6, pair_scale=pair_scale or 1.0, flags=kb.FLAG_WEIGHTS_STATIC)
    j.counter[0] = counter
    j.wait_counter = wait
    j.wait_target = target
    return j


def _weights(kernels, qtype, rows, k, tensor):
    n = rows * k // 256
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, n, kb.stream_key(77, tensor))
    return W


@pytest.mark.parametrize("qtype,rows,k", [(4, 4096, 4096), (6, 32000, 4096), (6, 300, 11008),
                                          (4, 1000, 8192), (5, 2048, 4096), (6, 100, 28672)])
def test_one_job_chain_equals_lone_matvec(kernels, qtype, rows, k):
    W = _weights(kernels, qtype, rows, k, qtype * 100 + rows % 97)
    x = torch.from_numpy(np.random.default_rng(rows).standard_normal(k).astype(np.float32)).cuda()
    y0 = torch.full((rows,), float("nan"), device="cuda")
    y1 = torch.full((rows,), float("nan"), device="cuda")
    mem = torch.zeros(2, dtype=torch.int64, device="cuda")  # epoch, counter
    kernels.matvec(qtype, y0, W, x, rows, k, 1)
    kernels.epoch_advance(mem.data_ptr())
    kernels.matvec_chain([_job(qtype, y1, W, x, rows, k, counter=mem.data_ptr() + 8)], mem.data_ptr())
    torch.cuda.synchronize()
    kernels.device_error()
    assert torch.equal(y0, y1)
    assert mem.tolist() == [1, rows]
    # and within the bound against the oracle
    y_ref, bound = oracle.matvec_ref(qtype, W.cpu().numpy(), x.cpu().numpy()[None, :], k, 0, rows)
    assert (np.abs(y1.cpu().numpy() - y_ref[0]) <= 1e-3 * bound[0]).all()


def test_three_job_chain_equals_three_launches_over_steps(kernels):
    """q|k|v -> o -> gate|up shaped like a 7B layer: x read by job 0, each later job reads the
    previous output after its counter; three steps with new input each (epoch 1, 2, 3)."""
    h, f = 4096, 11008
    Wqkv = _weights(kernels, 4, 3 * h, h, 1)
    Wo = _weights(kernels, 4, h, h, 2)
    Wgu = _weights(kernels, 4, 2 * f, h, 3)
    mem = torch.zeros(4, dtype=torch.int64, device="cuda")
    ep, c = mem.data_ptr(), mem.data_ptr() + 8
    qkv, o, a = (torch.zeros(n, device="cuda") for n in (3 * h, h, f))
    qkv2, o2, a2 = (torch.zeros(n, device="cuda") for n in (3 * h, h, f))
    x = torch.zeros(h, device="cuda")
    s = 1.0 / math.sqrt(f)
    jobs = [_job(4, qkv, Wqkv, x, 3 * h, h, counter=c, rmsnorm=True),
            _job(4, o, Wo, qkv, h, h, counter=c + 8, wait=c, target=3 * h),
            _job(4, a, Wgu, o, 2 * f, h, counter=c + 16, wait=c + 8, target=h, pair_scale=s)]
    for step in range(3):
        x.copy_(torch.from_numpy(np.random.default_rng(step).standard_normal(h).astype(np.float32)))
        kernels.epoch_advance(ep)
        kernels.matvec_chain(jobs, ep)
        kernels.matvec(4, qkv2, Wqkv, x, 3 * h, h, prologue=kb.PROLOGUE_RMSNORM, eps=1e-6)
        kernels.matvec(4, o2, Wo, qkv2, h, h)
        kernels.matvec(4, a2, Wgu, o2, 2 * f, h, epilogue=kb.EPILOGUE_PAIR_PRODUCT, pair_scale=s)
        torch.cuda.synchronize()
        kernels.device_error()
        assert torch.equal(qkv, qkv2) and torch.equal(o, o2) and torch.equal(a, a2), step
    assert mem.tolist() == [3, 3 * 3 * h, 3 * h, 3 * f]


def _stack_logits(kernels, cfg, xs, chain, graph=True):
    stream = torch.cuda.Stream()
    s = st.make_cuda_stack(cfg, kernels, stream=stream, chain=chain)
    out = []
    s.buf["x"].copy_(torch.from_numpy(xs[0]).cuda())
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        s.forward()
    torch.cuda.synchronize()
    out.append(s.buf["logits"].cpu().numpy())
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s.forward()
        for x in xs[1:]:
            s.buf["x"].copy_(torch.from_numpy(x).cuda())
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            out.append(s.buf["logits"].cpu().numpy())
        del g
    kernels.device_error()
    return out


@pytest.mark.parametrize("name,layers,exact", [("tiny", None, True), ("7b", 2, True), ("70b", 2, False)])
def test_chain_stack_equals_launch_per_projection_and_reference(kernels, name, layers, exact):
    """The chain stack's logits equal the launch-per-projection stack's bit for bit, except where a
    lone launch takes x in two parts (the 70B down projection, K = 28672: its partial sums are
    added in another order than the chain's), where they agree within 2e-5 of the largest logit;
    both within 1e-4 of it against the f64 reference."""
    cfg = st.CONFIGS[name] if layers is None else dataclasses.replace(st.CONFIGS[name], layers=layers)
    xs = [np.random.default_rng(11 + t).standard_normal(cfg.hidden).astype(np.float32) for t in range(3)]
    got = _stack_logits(kernels, cfg, xs, chain=True)
    base = _stack_logits(kernels, cfg, xs, chain=False)
    for t, x in enumerate(xs):
        if exact:
            assert np.array_equal(got[t], base[t]), f"token {t}"
        else:
            assert np.abs(got[t] - base[t]).max() <= 2e-5 * np.abs(base[t]).max(), f"token {t}"
        if t == 0:
            ref = st.reference_logits(cfg, x)
            assert np.abs(got[t] - ref).max() <= 1e-4 * np.abs(ref).max()


def test_chain_wait_that_is_never_met_gives_up(kernels):
    """A job waiting for a counter nothing adds to: the bounded wait runs out (about 2 s), the
    error word says so, and the context keeps working."""
    W = _weights(kernels, 4, 256, 4096, 5)
    x = torch.randn(4096, device="cuda")
    y = torch.zeros(256, device="cuda")
    mem = torch.zeros(3, dtype=torch.int64, device="cuda")
    kernels.epoch_advance(mem.data_ptr())
    job = _job(4, y, W, x, 256, 4096, counter=mem.data_ptr() + 8, wait=mem.data_ptr() + 16, target=1)
    kernels.matvec_chain([job], mem.data_ptr())
    torch.cuda.synchronize()
    with pytest.raises(kb.Error) as e:
        kernels.device_error()
    assert e.value.code == kb.KQ_E_DEVICE
    # the context still works
    y2 = torch.zeros(256, device="cuda")
    kernels.matvec(4, y2, W, x, 256, 4096)
    torch.cuda.synchronize()
    kernels.device_error()
    assert torch.isfinite(y2).all()


def test_chain_rejects_mixed_types_and_bad_arguments(kernels):
    W4 = _weights(kernels, 4, 16, 4096, 6)
    W6 = _weights(kernels, 6, 16, 4096, 7)
    x = torch.randn(4096, device="cuda")
    y = torch.zeros(16, device="cuda")
    mem = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(kb.Error) as e:
        kernels.matvec_chain([_job(4, y, W4, x, 16, 4096), _job(6, y, W6, x, 16, 4096)], mem.data_ptr())
    assert e.value.code == kb.KQ_E_INVALID
    with pytest.raises(kb.Error):
        kernels.matvec_chain([_job(4, y, W4, x, 16, 4096)] * 9, mem.data_ptr())
    with pytest.raises(kb.Error):
        kernels.matvec_chain([_job(4, y, W4, x, 16, 4096)], 0)
    j = _job(4, y, W4, x, 16, 4096)
    j.npush, j.push_rows = 2, 16  # push targets missing
    with pytest.raises(kb.Error):
        kernels.matvec_chain([j], mem.data_ptr())


def test_chain_pushing_to_its_own_full_vectors_over_steps(kernels):
    """The exchange form of a chain on one GPU (npush 1: outputs pushed to this GPU's own full
    vectors, counted with system-scope releases, waited for with system-scope acquires), three
    jobs a launch over four steps, against lone launches."""
    h, f = 4096, 11008
    Wqkv, Wo, Wgu = _weights(kernels, 4, 3 * h, h, 11), _weights(kernels, 4, h, h, 12), _weights(kernels, 4, 2 * f, h, 13)
    mem = torch.zeros(4, dtype=torch.int64, device="cuda")
    ep, c = mem.data_ptr(), mem.data_ptr() + 8
    loc = [torch.zeros(n, device="cuda") for n in (3 * h, h, f)]
    full = [torch.zeros(n, device="cuda") for n in (h, h, f)]
    r = [torch.zeros(n, device="cuda") for n in (3 * h, h, f)]
    x = torch.zeros(h, device="cuda")
    s = 1.0 / math.sqrt(f)
    jobs = [_job(4, loc[0], Wqkv, x, 3 * h, h, rmsnorm=True),
            _job(4, loc[1], Wo, full[0], h, h, wait=c, target=h),
            _job(4, loc[2], Wgu, full[1], 2 * f, h, wait=c + 8, target=h, pair_scale=s)]
    for i, (j, n) in enumerate(zip(jobs, (h, h, f))):
        j.npush, j.push_rows = 1, n
        j.push_y[0] = full[i].data_ptr()
        j.counter[0] = c + 8 * i
    for step in range(4):
        x.copy_(torch.from_numpy(np.random.default_rng(50 + step).standard_normal(h).astype(np.float32)))
        kernels.epoch_advance(ep)
        kernels.matvec_chain(jobs, ep)
        kernels.matvec(4, r[0], Wqkv, x, 3 * h, h, prologue=kb.PROLOGUE_RMSNORM, eps=1e-6)
        kernels.matvec(4, r[1], Wo, r[0], h, h)
        kernels.matvec(4, r[2], Wgu, r[1], 2 * f, h, epilogue=kb.EPILOGUE_PAIR_PRODUCT, pair_scale=s)
        torch.cuda.synchronize()
        kernels.device_error()
        assert torch.equal(full[0], r[0][:h]) and torch.equal(full[1], r[1]) and torch.equal(full[2], r[2]), step
    assert mem.tolist() == [4, 4 * h, 4 * h, 4 * f]
