"""Host-side logic of the row-sharded decode stack on CPU: shard plans, and world-size-2 and -4
gloo ranks running the stack on an oracle backend, against the unsharded reference."""
import math
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

from kernite_b200 import stack as st  # noqa: E402


class OracleBackend:
    """The stack's backend on the CPU oracle (test infrastructure): f64 matvecs of the
    f32-dequantised shard weights, gloo all-gathers."""

    def __init__(self, world: int):
        self.world = world

    def weights(self, shard, seed, tensor):
        key = oracle.stream_key(seed, tensor)
        nb = shard.k // 256
        return np.concatenate([oracle.fill(shard.qtype, key, r0 * nb, (r1 - r0) * nb) for r0, r1 in shard.runs])

    def vector(self, n):
        return torch.zeros(n, dtype=torch.float32)

    def matvec(self, W, shard, y, x, rmsnorm=False, eps=0.0, pair_scale=None, out=None, src=None):
        v = x.numpy().astype(np.float64)
        if rmsnorm:
            v = v / np.sqrt(np.mean(v * v) + eps)
        r, _ = oracle.matvec_ref(shard.qtype, W, v.astype(np.float32)[None, : shard.k], shard.k, 0, shard.rows)
        r = r[0]
        if pair_scale is not None:
            r = r[0::2] * r[1::2] * pair_scale
        y[: r.size] = torch.from_numpy(r.astype(np.float32))

    def gather(self, out, loc, part):
        a, b = part
        if self.world == 1:
            return
        parts = [torch.zeros(b - a, dtype=torch.float32) for _ in range(self.world)]
        dist.all_gather(parts, loc[a:b].contiguous())
        out.copy_(torch.cat(parts))


def test_plans_cover_every_row_once():
    for name, cfg in st.CONFIGS.items():
        for world in (1, 2, 4, 8):
            if cfg.kv % world or cfg.hidden % world or cfg.ffn % world or cfg.vocab % world:
                continue
            plans = [st.plan(cfg, r, world) for r in range(world)]
            for mname, qtype, rows, k in cfg.matrices() + [("head", 6, cfg.vocab, cfg.hidden)]:
                seen = np.zeros(rows, dtype=int)
                for p in plans:
                    for a, b in p[mname].runs:
                        seen[a:b] += 1
                assert (seen == 1).all(), (name, world, mname)
                assert all(p[mname].qtype == qtype and p[mname].k == k for p in plans)


def test_weight_bytes_match_baseline():
    assert st.CONFIGS["7b"].weight_bytes() == 4_122_255_360
    assert st.CONFIGS["70b"].weight_bytes() == 43_563_171_840


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = st.CONFIGS["tiny"]
        s = st.DecodeStack(cfg, OracleBackend(world), rank, world)
        x = np.random.default_rng(0).standard_normal(cfg.hidden).astype(np.float32)
        s.buf["x"].copy_(torch.from_numpy(x))
        s.forward()
        q.put((rank, s.buf["logits"].numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_unsharded_reference(world):
    cfg = st.CONFIGS["tiny"]
    x = np.random.default_rng(0).standard_normal(cfg.hidden).astype(np.float32)
    ref = st.reference_logits(cfg, x)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000 + 7 * world
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        np.testing.assert_allclose(out[r], ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
        np.testing.assert_array_equal(out[0], out[r])


def test_single_rank_oracle_backend_matches_reference():
    cfg = st.CONFIGS["tiny"]
    x = np.random.default_rng(1).standard_normal(cfg.hidden).astype(np.float32)
    s = st.DecodeStack(cfg, OracleBackend(1), 0, 1)
    s.buf["x"].copy_(torch.from_numpy(x))
    s.forward()
    ref = st.reference_logits(cfg, x)
    np.testing.assert_allclose(s.buf["logits"].numpy(), ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    assert s.launches_per_token() == 4 * cfg.layers + 1
    assert math.isfinite(float(np.abs(ref).max()))


def test_push_layout_and_targets():
    cfg = st.CONFIGS["70b"]
    off, total = st.push_layout(cfg)
    assert off["epoch"] == 40 and all(off[k] % 256 == 0 for k in st.FULL_KEYS)
    assert total >= off["logits"] + 4 * cfg.vocab
    # q is written once per layer: before token t's layer-L read the counter holds
    # (t-1) * layers * h from earlier tokens and (L+1) * h from this one
    mul, add = st.push_target(cfg, "q", 3)
    assert mul == cfg.layers * cfg.hidden and add == 3 * cfg.hidden
    assert st.push_target(cfg, "logits", 1) == (cfg.vocab, cfg.vocab)
