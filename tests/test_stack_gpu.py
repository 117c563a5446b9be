"""The decode stack on the GPU (libkq.so kernels) against the unsharded CPU reference, eager and
replayed from a CUDA graph. Multi-GPU sharding logic is covered by tests/test_stack_cpu.py
(gloo ranks); the NCCL path runs in bench.py under torchrun."""
import dataclasses

import numpy as np
import pytest
import torch

import oracle

from kernite_b200 import stack as st

pytestmark = pytest.mark.gpu


def head_bound(cfg, x_ref_last):
    """sum_k |w_head x| for the reference's normalised last activation (the 1e-3 bound)."""
    v = x_ref_last / np.sqrt(np.mean(x_ref_last ** 2) + cfg.eps)
    head = oracle.fill(6, oracle.stream_key(cfg.seed, cfg.tensor_id(cfg.layers, "head")), 0,
                       cfg.vocab * cfg.hidden // 256)
    _, bound = oracle.matvec_ref(6, head, v.astype(np.float32)[None, :], cfg.hidden, 0, cfg.vocab)
    return bound[0]


def run_stack(kernels, cfg, x, graph=False):
    s = st.make_cuda_stack(cfg, kernels)
    s.buf["x"].copy_(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    if graph:
        stream = torch.cuda.Stream()
        s.be.stream = stream
        with torch.cuda.stream(stream):
            s.forward()  # warm up outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s.forward()
        g.replay()
        torch.cuda.synchronize()
    else:
        s.forward()
        torch.cuda.synchronize()
    kernels.device_error()
    return s.buf["logits"].cpu().numpy()


def last_activation(cfg, x):
    """The reference's input to the head (its x after the last layer)."""
    c = dataclasses.replace(cfg)
    # recompute with the reference but stop before the head
    import math

    h, f, kv = c.hidden, c.ffn, c.kv
    xv = x.astype(np.float64)
    for layer in range(c.layers):
        xin = xv / np.sqrt(np.mean(xv * xv) + c.eps) if layer > 0 else xv

        def mv(name, qtype, rows, k, v):
            W = oracle.fill(qtype, oracle.stream_key(c.seed, c.tensor_id(layer, name)), 0, rows * k // 256)
            return oracle.matvec_ref(qtype, W, v.astype(np.float32)[None, :], k, 0, rows)[0][0]

        q = mv("qkv", 4, h + 2 * kv, h, xin)[:h]
        o = mv("o", 4, h, h, q)
        gu = mv("gate_up", 4, 2 * f, h, o)
        a = gu[0::2] * gu[1::2] / math.sqrt(f)
        xv = mv("down", 6, h, f, a)
    return xv


@pytest.mark.parametrize("graph", [False, True])
def test_tiny_stack_matches_reference(kernels, graph):
    cfg = st.CONFIGS["tiny"]
    x = np.random.default_rng(5).standard_normal(cfg.hidden).astype(np.float32)
    got = run_stack(kernels, cfg, x, graph=graph)
    ref = st.reference_logits(cfg, x)
    bound = head_bound(cfg, last_activation(cfg, x))
    assert (np.abs(got - ref) <= 1e-3 * bound).all()


def test_7b_shapes_two_layers_match_reference(kernels):
    cfg = dataclasses.replace(st.CONFIGS["7b"], layers=2)
    x = np.random.default_rng(7).standard_normal(cfg.hidden).astype(np.float32)
    got = run_stack(kernels, cfg, x, graph=True)
    ref = st.reference_logits(cfg, x)
    bound = head_bound(cfg, last_activation(cfg, x))
    assert (np.abs(got - ref) <= 1e-3 * bound).all()


def test_graph_replay_equals_eager(kernels):
    cfg = st.CONFIGS["tiny"]
    x = np.random.default_rng(9).standard_normal(cfg.hidden).astype(np.float32)
    a = run_stack(kernels, cfg, x, graph=False)
    b = run_stack(kernels, cfg, x, graph=True)
    assert np.array_equal(a, b)
