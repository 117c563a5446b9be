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

    def kv_cache(self, cfg, world):
        return ([], [])

    def attend(self, stack, layer, pos):
        cfg, b, w = stack.cfg, stack.buf, self.world
        nh, nkv, d = cfg.n_heads // w, cfg.n_kv // w, cfg.head_dim
        q, k, v = oracle.rope_ref(b["qkv"].numpy(), nh, nkv, d, pos, cfg.rope_base)
        K, V = stack.caches[layer]
        K.append(k.astype(np.float32).astype(np.float16))
        V.append(v.astype(np.float32).astype(np.float16))
        att, _ = oracle.attention_ref(q.astype(np.float32), np.stack(K), np.stack(V), nh, nkv, d, pos + 1)
        b["att"][:] = torch.from_numpy(att.reshape(-1).astype(np.float32))

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


ATT_TINY = __import__("dataclasses").replace(st.CONFIGS["tiny"], attention=True, max_pos=8)


def _rank(rank, world, port, q, attention=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ATT_TINY if attention else st.CONFIGS["tiny"]
        s = st.DecodeStack(cfg, OracleBackend(world), rank, world)
        outs = []
        for t in range(3 if attention else 1):
            x = np.random.default_rng(t).standard_normal(cfg.hidden).astype(np.float32)
            s.buf["x"].copy_(torch.from_numpy(x))
            s.forward()
            outs.append(s.buf["logits"].numpy().copy())
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,attention", [(2, False), (4, False), (2, True)])
def test_gloo_ranks_match_unsharded_reference(world, attention):
    """Sharded ranks against the unsharded reference; with attention, three tokens in a row
    (each rank attends over its own heads' caches, the attention outputs gathered for o)."""
    cfg = ATT_TINY if attention else st.CONFIGS["tiny"]
    cache = {}
    refs = [st.reference_logits(cfg, np.random.default_rng(t).standard_normal(cfg.hidden).astype(np.float32),
                                cache=cache) for t in range(3 if attention else 1)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000 + 7 * world + (3 if attention else 0)
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, attention)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        for t, ref in enumerate(refs):
            np.testing.assert_allclose(out[r][t], ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
            np.testing.assert_array_equal(out[0][t], out[r][t])


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


def test_push_splits_only_short_shards_with_several_k_tiles():
    c70, c7 = st.CONFIGS["70b"], st.CONFIGS["7b"]
    assert st.push_splits(c70, 1, 148) == {"q": 1, "o": 1, "xd": 1}
    assert st.push_splits(c70, 2, 148) == {"q": 1, "o": 1, "xd": 1}
    assert st.push_splits(c70, 8, 148) == {"q": 1, "o": 2, "xd": 2}
    assert st.push_splits(c7, 8, 148)["o"] == 1  # k = 4096: one K-tile a row, nothing to split
    off, total = st.push_layout(c70, st.push_splits(c70, 8, 148))
    assert off["a"] - off["o"] >= 2 * c70.hidden * 8 and off["o"] - off["q"] >= c70.hidden * 8


def test_push_layout_and_tags():
    cfg = st.CONFIGS["70b"]
    off, total = st.push_layout(cfg)
    assert off["epoch"] == 0 and all(off[k] % 256 == 0 and off[k] >= 256 for k in st.FULL_KEYS)
    ends = sorted((off[k], off[k] + 8 * n) for k, n in st.full_sizes(cfg).items())
    assert all(ends[i][1] <= ends[i + 1][0] for i in range(len(ends) - 1)) and ends[-1][1] <= total
    # every write of a vector over several tokens carries its own tag, never 0, and the reader of
    # each write expects exactly the writer's tag
    for key in st.FULL_KEYS:
        writes = 1 if key == "logits" else cfg.layers
        tags = []
        for t in range(1, 4):
            for occ in range(1, writes + 1):
                mul, add = st.push_tag(cfg, key, occ)
                tags.append((t - 1) * mul + add)
        assert len(set(tags)) == len(tags) and min(tags) >= 1


# ---------------------------------------------------------------- chains (host logic)

ALIAS_ONE_RANK = {"q": "qkv", "o": "o_loc", "a": "a_loc", "xd": "x_loc", "logits": "l_loc"}


def _simulate_chain(cfg, world, tokens=3):
    """Runs the token's chain jobs on `world` simulated ranks, job after job, tagging every
    element each job stores (local output, pushes into every rank's full vectors) and adding to
    the counters as the kernel does; before a job reads x on a rank, its wait must already be
    met and every element of x must hold this token's output of the job it waits for."""
    plans = [st.chain_plan(cfg, r, world) for r in range(world)]
    jobs0, launches = plans[0]
    sizes = st.full_sizes(cfg)
    for r in range(world):
        assert [(j.name, j.layer, j.counter, j.wait, j.wait_target) for j in plans[r][0]] == \
               [(j.name, j.layer, j.counter, j.wait, j.wait_target) for j in jobs0]
    counters = [np.zeros(len(jobs0), dtype=np.int64) for _ in range(world)]
    full = [{k: np.full(n, -1, dtype=np.int64) for k, n in sizes.items()} for _ in range(world)]
    local = [{} for _ in range(world)]
    for t in range(1, tokens + 1):
        tag = lambda i: t * 100000 + i
        for r in range(world):
            full[r]["x"] = np.full(cfg.hidden, tag(-1))  # the token's input, on every rank
        for i, j0 in enumerate(jobs0):
            for r in range(world):
                j = plans[r][0][i]
                if j.wait is not None:
                    assert counters[r][j.wait] >= t * j.wait_target, (t, j.name, j.layer, r)
                    want = tag(j.wait)
                else:
                    want = tag(-1)
                if world == 1 and j.x in ALIAS_ONE_RANK:
                    src = local[r][ALIAS_ONE_RANK[j.x]][: sizes[j.x]]
                else:
                    src = full[r][j.x]
                assert src.size >= j.k and (src[: j.k] == want).all(), (t, j.name, j.layer, r)
            for r in range(world):
                j = plans[r][0][i]
                local[r][j.y] = np.full(j.outputs, tag(i))
                if world == 1:
                    counters[r][j.counter] += j.outputs
                else:
                    assert j.push_rows <= j.outputs
                    for p in range(world):
                        dst = full[p][j.push][r * j.push_rows:(r + 1) * j.push_rows]
                        assert dst.size == j.push_rows
                        dst[:] = tag(i)
                        counters[p][j.counter] += j.push_rows
        head = len(jobs0) - 1
        for r in range(world):
            logits = local[r]["l_loc"] if world == 1 else full[r]["logits"]
            assert (logits == tag(head)).all()
    return jobs0, launches


@pytest.mark.parametrize("name,world", [("tiny", 1), ("tiny", 2), ("tiny", 4), ("7b", 1), ("7b", 2),
                                        ("7b", 8), ("70b", 1), ("70b", 8)])
def test_chain_plan_orders_every_read_after_its_writes(name, world):
    cfg = st.CONFIGS[name]
    if name != "tiny":
        cfg = __import__("dataclasses").replace(cfg, layers=3)
    jobs, launches = _simulate_chain(cfg, world)
    assert sorted(i for l in launches for i in l) == list(range(len(jobs)))
    for l in launches:
        assert 1 <= len(l) <= 8 and l == list(range(l[0], l[0] + len(l)))
        assert len({(jobs[i].qtype, jobs[i].k) for i in l}) == 1
    # per layer: q|k|v, o, gate|up in one launch, down in another; then the head
    assert [len(l) for l in launches] == [3, 1] * cfg.layers + [1]


def test_chain_layout_fits_counters_and_vectors():
    for name, cfg in st.CONFIGS.items():
        n = len(st.chain_plan(cfg, 0, 1)[0])
        off, total = st.chain_layout(cfg, n)
        assert off["counters"] == 8 and off["epoch"] == 0
        ends = sorted((off[k], off[k] + 4 * v) for k, v in st.full_sizes(cfg).items())
        assert ends[0][0] >= 8 + 8 * n and all(a % 256 == 0 for a, _ in ends)
        assert all(ends[i][1] <= ends[i + 1][0] for i in range(len(ends) - 1)) and ends[-1][1] <= total
