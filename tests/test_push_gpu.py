"""kq_matvec_push on one GPU, pushing to its own full vector (npush 1): the warp-MMA push kernel's
outputs equal the lone launch's bit for bit, both in y and in the full vector; the counter gains
the pushed count; a second launch waits for that count before it reads x; and the CUDA-core push
(KQ_FLAG_CUDA_CORES) agrees within the bound. The exchange between GPUs is covered by
tests/test_stack_multigpu.py."""
import numpy as np
import pytest
import torch

import oracle

import kernite_b200 as kb

pytestmark = pytest.mark.gpu


def _w(kernels, qtype, rows, k, t):
    n = rows * k // 256
    W = torch.empty(n * kb.block_bytes(qtype), dtype=torch.uint8, device="cuda")
    kernels.fill(qtype, W, 0, n, kb.stream_key(55, t))
    return W


def _desc(npush, push_rows, full, counter, wait=0, epoch=0, mul=0, add=0):
    d = kb.KqPushDesc()
    d.npush, d.push_rows = npush, push_rows
    d.y[0] = full
    d.counter[0] = counter
    d.wait_counter, d.epoch, d.wait_mul, d.wait_add = wait, epoch, mul, add
    return d


@pytest.mark.parametrize("qtype,rows,k,pair", [(4, 4096, 4096, False), (6, 32000, 4096, False),
                                               (4, 2048, 8192, True), (6, 300, 11008, False),
                                               (5, 1024, 4096, False), (6, 4096, 28672, False)])
def test_push_kernel_equals_lone_kernel(kernels, qtype, rows, k, pair):
    W = _w(kernels, qtype, rows, k, rows)
    x = torch.from_numpy(np.random.default_rng(rows).standard_normal(k).astype(np.float32)).cuda()
    outs = rows // 2 if pair else rows
    kw = dict(epilogue=kb.EPILOGUE_PAIR_PRODUCT if pair else kb.EPILOGUE_NONE, pair_scale=0.03)
    y0 = torch.full((outs,), float("nan"), device="cuda")
    y1 = torch.full((outs,), float("nan"), device="cuda")
    full = torch.full((outs + 7,), float("nan"), device="cuda")
    mem = torch.zeros(2, dtype=torch.int64, device="cuda")
    push_rows = outs - 5 if outs > 5 else outs
    kernels.matvec(qtype, y0, W, x, rows, k, 1, **kw)
    kernels.matvec_push(qtype, y1, W, x, rows, k, _desc(1, push_rows, full.data_ptr() + 8, mem.data_ptr()), **kw)
    torch.cuda.synchronize()
    kernels.device_error()
    assert torch.equal(y0, y1)
    assert torch.equal(full[2:2 + push_rows], y0[:push_rows])
    assert torch.isnan(full[:2]).all() and torch.isnan(full[2 + push_rows:]).all()
    assert int(mem[0]) == push_rows


def test_push_waits_for_the_count_before_reading_x(kernels):
    """Two pushes in a row over three steps: the second reads the first's full vector after its
    counter reaches step * rows ((epoch - 1) * mul + add)."""
    h = 4096
    W1, W2 = _w(kernels, 4, h, h, 1), _w(kernels, 4, h, h, 2)
    mem = torch.zeros(3, dtype=torch.int64, device="cuda")  # epoch, counter 1, counter 2
    ep, c1, c2 = mem.data_ptr(), mem.data_ptr() + 8, mem.data_ptr() + 16
    x = torch.zeros(h, device="cuda")
    y1, y2, full1, full2 = (torch.zeros(h, device="cuda") for _ in range(4))
    r1, r2 = torch.zeros(h, device="cuda"), torch.zeros(h, device="cuda")
    for step in range(1, 4):
        x.copy_(torch.from_numpy(np.random.default_rng(step).standard_normal(h).astype(np.float32)))
        mem[0] += 1
        kernels.matvec_push(4, y1, W1, x, h, h, _desc(1, h, full1.data_ptr(), c1))
        kernels.matvec_push(4, y2, W2, full1, h, h, _desc(1, h, full2.data_ptr(), c2, wait=c1, epoch=ep,
                                                          mul=h, add=h))
        kernels.matvec(4, r1, W1, x, h, h, 1)
        kernels.matvec(4, r2, W2, r1, h, h, 1)
        torch.cuda.synchronize()
        kernels.device_error()
        assert torch.equal(full2, r2), step
    assert mem.tolist() == [3, 3 * h, 3 * h]


def test_cuda_core_push_agrees_within_the_bound(kernels):
    rows, k = 1024, 4096
    W = _w(kernels, 6, rows, k, 3)
    xh = np.random.default_rng(4).standard_normal(k).astype(np.float32)
    x = torch.from_numpy(xh).cuda()
    y, full = torch.zeros(rows, device="cuda"), torch.zeros(rows, device="cuda")
    mem = torch.zeros(1, dtype=torch.int64, device="cuda")
    kernels.matvec_push(6, y, W, x, rows, k, _desc(1, rows, full.data_ptr(), mem.data_ptr()),
                        flags=kb.FLAG_CUDA_CORES)
    torch.cuda.synchronize()
    kernels.device_error()
    ref, bound = oracle.matvec_ref(6, W.cpu().numpy(), xh[None, :], k, 0, rows)
    assert (np.abs(full.cpu().numpy() - ref[0]) <= 1e-3 * bound[0]).all()
    assert torch.equal(full, y) and int(mem[0]) == rows


def test_tagged_push_chain_of_two_over_steps(kernels):
    """The tagged exchange on one GPU: the first launch pushes its outputs as (value, tag) pairs
    into a tagged full vector, the second reads that vector waiting on each element's tag and
    pushes its own; kq_tagged_unpack gives the plain values. Three steps: the tags advance with
    the epoch, so a step never reads the previous step's elements."""
    h = 4096
    W1, W2 = _w(kernels, 4, h, h, 21), _w(kernels, 6, h, h, 22)
    mem = torch.zeros(1, dtype=torch.int64, device="cuda")  # epoch
    ep = mem.data_ptr()
    x = torch.zeros(h, device="cuda")
    y1, y2 = torch.zeros(h, device="cuda"), torch.zeros(h, device="cuda")
    t1 = torch.zeros(2 * h, device="cuda")  # tagged: 8 bytes an element
    t2 = torch.zeros(2 * h, device="cuda")
    plain = torch.full((h,), float("nan"), device="cuda")
    r1, r2 = torch.zeros(h, device="cuda"), torch.zeros(h, device="cuda")
    for step in range(1, 4):
        x.copy_(torch.from_numpy(np.random.default_rng(step).standard_normal(h).astype(np.float32)))
        mem[0] += 1
        d1 = _desc(1, h, t1.data_ptr(), 0, epoch=ep)
        d1.flags, d1.push_mul, d1.push_add = kb.PUSH_TAGGED, 1, 1
        kernels.matvec_push(4, y1, W1, x, h, h, d1)
        d2 = _desc(1, h, t2.data_ptr(), 0, epoch=ep, mul=1, add=1)
        d2.flags, d2.push_mul, d2.push_add = kb.PUSH_TAGGED | kb.PUSH_TAGGED_X, 1, 1
        kernels.matvec_push(6, y2, W2, t1, h, h, d2, prologue=kb.PROLOGUE_RMSNORM, eps=1e-6)
        kernels.tagged_unpack(plain, t2, h, ep, 1, 1)
        kernels.matvec(4, r1, W1, x, h, h, 1)
        kernels.matvec(6, r2, W2, r1, h, h, 1, prologue=kb.PROLOGUE_RMSNORM, eps=1e-6)
        torch.cuda.synchronize()
        kernels.device_error()
        assert torch.equal(y1, r1) and torch.equal(y2, r2) and torch.equal(plain, r2), step
        tags = t2.view(torch.int32)[1::2]
        assert (tags == step).all()


def test_tagged_push_into_a_long_k_matvec(kernels):
    """A tagged vector of 28672 elements read by a Q6_K matvec of the 70B down projection's
    2-way shard shape (4096 x 28672), whose x table is the whole of x (the lone launch of that
    shape takes x in two parts, so its sums run in another order). Two steps: the first launch
    equals its lone launch bit for bit, the second agrees with its lone launch and with the oracle
    within the bound, and its pushed vector equals its own outputs."""
    h, f = 4096, 28672
    W1, W2 = _w(kernels, 4, f, h, 31), _w(kernels, 6, h, f, 32)
    mem = torch.zeros(1, dtype=torch.int64, device="cuda")  # epoch
    ep = mem.data_ptr()
    x = torch.zeros(h, device="cuda")
    y1, y2 = torch.zeros(f, device="cuda"), torch.zeros(h, device="cuda")
    t1, t2 = torch.zeros(2 * f, device="cuda"), torch.zeros(2 * h, device="cuda")
    plain = torch.full((h,), float("nan"), device="cuda")
    r1, r2 = torch.zeros(f, device="cuda"), torch.zeros(h, device="cuda")
    for step in range(1, 3):
        x.copy_(torch.from_numpy(np.random.default_rng(40 + step).standard_normal(h).astype(np.float32)))
        mem[0] += 1
        d1 = _desc(1, f, t1.data_ptr(), 0, epoch=ep)
        d1.flags, d1.push_mul, d1.push_add = kb.PUSH_TAGGED, 1, 1
        kernels.matvec_push(4, y1, W1, x, f, h, d1)
        d2 = _desc(1, h, t2.data_ptr(), 0, epoch=ep, mul=1, add=1)
        d2.flags, d2.push_mul, d2.push_add = kb.PUSH_TAGGED | kb.PUSH_TAGGED_X, 1, 1
        kernels.matvec_push(6, y2, W2, t1, h, f, d2)
        kernels.tagged_unpack(plain, t2, h, ep, 1, 1)
        kernels.matvec(4, r1, W1, x, f, h, 1)
        kernels.matvec(6, r2, W2, r1, h, f, 1)
        torch.cuda.synchronize()
        kernels.device_error()
        assert torch.equal(y1, r1) and torch.equal(plain, y2), step
        _, bound = oracle.matvec_ref(6, W2.cpu().numpy(), np.abs(r1.cpu().numpy())[None, :], f, 0, h)
        assert (np.abs(y2.cpu().numpy() - r2.cpu().numpy()) <= 2e-3 * bound[0]).all(), step
    ref, bound = oracle.matvec_ref(6, W2.cpu().numpy(), r1.cpu().numpy()[None, :], f, 0, 64)
    assert (np.abs(y2.cpu().numpy()[:64] - ref[0]) <= 1e-3 * bound[0]).all()


def test_tagged_read_of_a_stale_vector_gives_up(kernels):
    """x whose elements carry an old tag: the bounded wait runs out (about 2 s), the error word
    says so, and the context keeps working."""
    h = 1024
    W = _w(kernels, 4, 256, h, 23)
    mem = torch.ones(1, dtype=torch.int64, device="cuda")
    stale = torch.zeros(2 * h, device="cuda")  # tags 0: never this step's
    y = torch.zeros(256, device="cuda")
    d = _desc(1, 256, torch.zeros(512, device="cuda").data_ptr(), 0, epoch=mem.data_ptr(), mul=1, add=1)
    d.flags, d.push_mul, d.push_add = kb.PUSH_TAGGED | kb.PUSH_TAGGED_X, 1, 1
    kernels.matvec_push(4, y, W, stale, 256, h, d)
    torch.cuda.synchronize()
    with pytest.raises(kb.Error) as e:
        kernels.device_error()
    assert e.value.code == kb.KQ_E_DEVICE
    kernels.matvec(4, y, W, torch.zeros(h, device="cuda"), 256, h, 1)
    torch.cuda.synchronize()
    kernels.device_error()


def test_split_k_pushes_slots_the_reader_adds_up(kernels):
    """Split K (ksplit 2): CTA pairs each multiply half of a row's K-tiles and push their partial
    sums into their own slot of the tagged vector; the next launch (x_slots 2) reads every element
    as the sum of its two slots. The slots add up to the unsplit matvec within the bound, the
    reader's outputs are the matvec of that sum, and a second run gives the same bits."""
    rows1, k1, rows2 = 2048, 8192, 1024
    W1, W2 = _w(kernels, 4, rows1, k1, 31), _w(kernels, 6, rows2, rows1, 32)
    mem = torch.ones(1, dtype=torch.int64, device="cuda")
    ep = mem.data_ptr()
    xh = np.random.default_rng(9).standard_normal(k1).astype(np.float32)
    x = torch.from_numpy(xh).cuda()
    outs = []
    for run in range(2):
        t1 = torch.zeros(2 * 2 * rows1, device="cuda")  # 2 slots, 8 bytes an element
        t2 = torch.zeros(2 * rows2, device="cuda")
        d1 = _desc(1, rows1, t1.data_ptr(), 0, epoch=ep)
        d1.flags, d1.push_mul, d1.push_add, d1.ksplit = kb.PUSH_TAGGED, 1, 1, 2
        kernels.matvec_push(4, torch.zeros(rows1, device="cuda"), W1, x, rows1, k1, d1)
        d2 = _desc(1, rows2, t2.data_ptr(), 0, epoch=ep, mul=1, add=1)
        d2.flags, d2.push_mul, d2.push_add, d2.x_slots = kb.PUSH_TAGGED | kb.PUSH_TAGGED_X, 1, 1, 2
        y2 = torch.zeros(rows2, device="cuda")
        kernels.matvec_push(6, y2, W2, t1, rows2, rows1, d2)
        torch.cuda.synchronize()
        kernels.device_error()
        slots = t1.view(2, rows1, 2)[:, :, 0].cpu().numpy().astype(np.float64)
        assert (t1.view(torch.int32)[1::2] == 1).all()
        outs.append((slots.sum(0), y2.cpu().numpy()))
    ref1, b1 = oracle.matvec_ref(4, W1.cpu().numpy(), xh[None, :], k1, 0, rows1)
    assert (np.abs(outs[0][0] - ref1[0]) <= 1e-3 * b1[0]).all()
    x2 = outs[0][0].astype(np.float32)
    ref2, b2 = oracle.matvec_ref(6, W2.cpu().numpy(), x2[None, :], rows1, 0, rows2)
    assert (np.abs(outs[0][1] - ref2[0]) <= 1e-3 * b2[0]).all()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
