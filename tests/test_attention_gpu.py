"""A decode step's attention on the GPU (kq_rope_append, kq_attention_decode) against the f64
restatements in oracle/: rotary embedding of q and k at early and very late positions with the
Llama 2 and Llama 3 bases, the f16 cache rows it appends, grouped-query attention over caches of
1 to 4096 positions with 1 to 16 query heads per key/value head, and a few steps in a row, each
appending to the cache and attending over it. Outputs within 1e-3 * sum_p w_p |v_p| (the
tolerance of the matvecs, with the values in place of w x)."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _f16(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16)


@pytest.mark.parametrize("nh,nkv,d,pos,base", [(32, 32, 128, 0, 1e4), (32, 32, 128, 1, 1e4),
                                               (64, 8, 128, 4095, 5e5), (8, 2, 64, 100000, 1e4),
                                               (4, 1, 256, 77, 5e5)])
def test_rope_append_matches_the_rotation(kernels, nh, nkv, d, pos, base):
    rng = np.random.default_rng(pos + d)
    qkv = rng.standard_normal((nh + 2 * nkv) * d).astype(np.float32)
    cap = pos + 2
    kc = torch.zeros(cap * nkv * d, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q_out = torch.full((nh * d,), float("nan"), device="cuda")
    kernels.rope_append(torch.from_numpy(qkv).cuda(), q_out, kc, vc, nh, nkv, d, pos, base)
    torch.cuda.synchronize()
    kernels.device_error()
    q, k, v = oracle.rope_ref(qkv, nh, nkv, d, pos, base)
    got_q = q_out.cpu().numpy().astype(np.float64).reshape(nh, d)
    assert np.abs(got_q - q).max() <= 2 ** -22 * max(1.0, np.abs(q).max())
    row = slice(pos * nkv * d, (pos + 1) * nkv * d)
    got_k = kc[row].cpu().numpy().astype(np.float64).reshape(nkv, d)
    # f16 of the f64 rotation: equal, or one f16 step apart where the f64 value sits on a tie
    assert (np.abs(got_k - _f16(k).astype(np.float64)) <= np.abs(k) * 2 ** -10 + 2 ** -24).all()
    assert np.array_equal(vc[row].cpu().numpy(), _f16(v).reshape(-1))
    # nothing written outside row pos
    assert not kc[: pos * nkv * d].any() and not kc[(pos + 1) * nkv * d:].any()


@pytest.mark.parametrize("nh,nkv,d,length", [(32, 32, 128, 1), (32, 32, 128, 300), (64, 8, 128, 4096),
                                             (8, 1, 64, 77), (16, 2, 256, 2000), (32, 2, 128, 1025),
                                             (8, 8, 128, 33)])
def test_attention_matches_the_oracle(kernels, nh, nkv, d, length):
    rng = np.random.default_rng(length * 7 + nh)
    q = (rng.standard_normal(nh * d) * 0.5).astype(np.float32)
    K = _f16(rng.standard_normal((length, nkv, d)))
    V = _f16(rng.standard_normal((length, nkv, d)))
    kc = torch.from_numpy(K.reshape(-1)).cuda()
    vc = torch.from_numpy(V.reshape(-1)).cuda()
    out = torch.full((nh * d,), float("nan"), device="cuda")
    wb = kernels.attention_workspace(nh, nkv, d, length)
    ws = torch.empty(wb // 4 + 4, dtype=torch.float32, device="cuda")
    kernels.attention(out, torch.from_numpy(q).cuda(), kc, vc, nh, nkv, d, length, ws, wb)
    torch.cuda.synchronize()
    kernels.device_error()
    ref, bound = oracle.attention_ref(q, K, V, nh, nkv, d, length)
    got = out.cpu().numpy().astype(np.float64).reshape(nh, d)
    assert np.isfinite(got).all()
    assert (np.abs(got - ref) <= 1e-3 * bound + 1e-7).all(), np.abs(got - ref).max()


def test_decode_steps_append_and_attend(kernels):
    """Eight steps of one layer's attention: each step's q|k|v is rotated at its position, its k
    and v appended, and its q attends over every position so far."""
    nh, nkv, d, steps, base = 16, 4, 128, 8, 1e4
    kc = torch.zeros(steps * nkv * d, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    ws = torch.empty(kernels.attention_workspace(nh, nkv, d, steps) // 4 + 4, device="cuda")
    K = np.zeros((steps, nkv, d))
    V = np.zeros((steps, nkv, d))
    for pos in range(steps):
        qkv = np.random.default_rng(pos).standard_normal((nh + 2 * nkv) * d).astype(np.float32)
        q_out = torch.empty(nh * d, device="cuda")
        out = torch.empty(nh * d, device="cuda")
        kernels.rope_append(torch.from_numpy(qkv).cuda(), q_out, kc, vc, nh, nkv, d, pos, base)
        kernels.attention(out, q_out, kc, vc, nh, nkv, d, pos + 1, ws, ws.numel() * 4)
        torch.cuda.synchronize()
        q, k, v = oracle.rope_ref(qkv, nh, nkv, d, pos, base)
        K[pos], V[pos] = _f16(k), _f16(v)
        ref, bound = oracle.attention_ref(q_out.cpu().numpy(), K, V, nh, nkv, d, pos + 1)
        got = out.cpu().numpy().astype(np.float64).reshape(nh, d)
        assert (np.abs(got - ref) <= 1e-3 * bound + 1e-7).all(), pos
    kernels.device_error()


def test_attention_rejects_bad_shapes_and_a_short_workspace(kernels):
    import kernite_b200 as kb

    q = torch.zeros(64 * 128, device="cuda")
    kc = torch.zeros(16 * 8 * 128, dtype=torch.float16, device="cuda")
    ws = torch.zeros(16, device="cuda")
    with pytest.raises(kb.Error):
        kernels.attention(q, q, kc, kc, 64, 3, 128, 16, ws, 64)  # 64 heads over 3 kv heads
    with pytest.raises(kb.Error):
        kernels.attention(q, q, kc, kc, 64, 8, 128, 16, ws, 64)  # workspace too small
    with pytest.raises(kb.Error):
        kernels.attention(q, q, kc, kc, 64, 2, 128, 16, ws, 1 << 20)  # 32 heads a group


@pytest.mark.parametrize("name,layers", [("tiny", None), ("7b", 2), ("70b", 1)])
def test_stack_with_attention_matches_reference_over_tokens(kernels, name, layers):
    """A real decode step (q|k|v, RoPE, cache append, GQA attention, o, gate|up, down; the head)
    for four tokens in a row on one GPU against the f64 reference carrying its own caches."""
    import dataclasses

    from kernite_b200 import stack as st

    cfg = dataclasses.replace(st.CONFIGS[name], attention=True, max_pos=8)
    if layers is not None:
        cfg = dataclasses.replace(cfg, layers=layers)
    s = st.make_cuda_stack(cfg, kernels)
    cache = {}
    for t in range(4):
        x = np.random.default_rng(40 + t).standard_normal(cfg.hidden).astype(np.float32)
        s.buf["x"].copy_(torch.from_numpy(x).cuda())
        s.forward()
        torch.cuda.synchronize()
        got = s.buf["logits"].cpu().numpy().astype(np.float64)
        ref = st.reference_logits(cfg, x, cache=cache)
        assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), t
    kernels.device_error()
    assert s.pos == 4
