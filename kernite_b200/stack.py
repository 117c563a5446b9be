"""Llama-shaped decode matvec stacks (BASELINE configs 2 and 4), row-sharded over N ranks.

Per layer, with hidden h, FFN f, K/V width kv (grouped-query attention):

    q|k|v = W_qkv . n(x)          (rows h + 2 kv; k and v are computed and not consumed)
    o     = W_o . q
    a     = (W_gate . o) * (W_up . o) / sqrt(f)     (W_gate and W_up rows interleaved)
    x'    = W_down . a
    logits = W_head . n(x_last)

where n(x) = x / sqrt(mean(x^2) + eps) is applied to every layer input but the first (so each
layer sees the RMS-normalised output of the previous one) and to the head's input. Attention
itself, RoPE and the KV cache are not part of this matvec stack. Q/K/V/O and gate/up are
Q4_K; down and the head are Q6_K. Each projection is one matvec launch with its elementwise
glue fused: the RMS norm as the kernel prologue, the gate*up product as its epilogue.

Sharding (one process per GPU): rank g of N holds rows [g R/N, (g+1) R/N) of every matrix
(for W_qkv: that slice of each of the q, k and v parts; for gate/up: that slice of the row
pairs). After each projection an all-gather of the f32 output slices rebuilds the full
vector on every rank: q, o, a, x' (4 per layer) and the logits. The synthetic weights of a
shard are exactly those rows of the unsharded model (the generator is counter-based), so any
N computes the same logits.

The math runs on a backend: :class:`CudaBackend` (libkq.so kernels, torch.distributed /
NCCL all-gathers, optional CUDA-graph capture of a whole token) is the product; tests plug in
a CPU backend built on the oracle to check the sharding and gather logic with gloo ranks.
Kernite has no decode stack; the shape of `forward` follows its microgpt forward pass
(examples/microgpt/src/model.rs:294-308), where each layer is a chain of matmul launches.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

QK = 256
BLOCK_BYTES = {4: 144, 6: 210}


@dataclass(frozen=True)
class StackConfig:
    name: str
    layers: int
    hidden: int
    ffn: int
    kv: int      # width of each of K and V
    vocab: int
    eps: float = 1e-6
    seed: int = 2026
    # A real decode step's attention between q|k|v and o (off for BASELINE's matvec stacks):
    # the q and k heads rotated at the step's position (RoPE), k and v appended to a per-layer
    # f16 cache of `max_pos` positions, and o = W_o . attention(q, cache) instead of W_o . q.
    attention: bool = False
    head_dim: int = 128
    rope_base: float = 10000.0
    max_pos: int = 64

    @property
    def n_heads(self) -> int:
        return self.hidden // self.head_dim

    @property
    def n_kv(self) -> int:
        return self.kv // self.head_dim

    def matrices(self):
        """(name, qtype, rows, k) of one layer's matrices, then the head."""
        h, f, kv = self.hidden, self.ffn, self.kv
        return [("qkv", 4, h + 2 * kv, h), ("o", 4, h, h), ("gate_up", 4, 2 * f, h),
                ("down", 6, h, f)]

    def weight_bytes(self) -> int:
        per_layer = sum(rows * (k // QK) * BLOCK_BYTES[q] for _, q, rows, k in self.matrices())
        return self.layers * per_layer + self.vocab * (self.hidden // QK) * BLOCK_BYTES[6]

    def tensor_id(self, layer: int, name: str) -> int:
        names = ["qkv", "o", "gate_up", "down", "head"]
        return layer * 8 + names.index(name)


CONFIGS = {
    "7b": StackConfig("llama-7b (BASELINE configs[2])", 32, 4096, 11008, 4096, 32000),
    "70b": StackConfig("llama-70b (BASELINE configs[4])", 80, 8192, 28672, 1024, 32000),
    # small shapes for tests
    "tiny": StackConfig("tiny", 2, 512, 1024, 256, 1000),
}


@dataclass
class Shard:
    """The rows a rank holds of one matrix: list of (global_row_start, global_row_end) runs, in
    local order, and the slice of the output that is gathered."""
    qtype: int
    k: int
    runs: list[tuple[int, int]]
    gathered: tuple[int, int] = (0, 0)  # local output rows that feed the all-gather

    @property
    def rows(self) -> int:
        return sum(b - a for a, b in self.runs)

    @property
    def nbytes(self) -> int:
        return self.rows * (self.k // QK) * BLOCK_BYTES[self.qtype]


def split(n: int, rank: int, world: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"{n} rows do not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def plan(cfg: StackConfig, rank: int, world: int) -> dict[str, Shard]:
    """The row shards rank `rank` of `world` holds, per matrix of a layer and the head."""
    h, f, kv = cfg.hidden, cfg.ffn, cfg.kv
    q0, q1 = split(h, rank, world)
    k0, k1 = split(kv, rank, world)
    f0, f1 = split(f, rank, world)
    v0, v1 = split(cfg.vocab, rank, world)
    qkv = Shard(4, h, [(q0, q1), (h + k0, h + k1), (h + kv + k0, h + kv + k1)], (0, q1 - q0))
    o = Shard(4, h, [(q0, q1)], (0, q1 - q0))
    gate_up = Shard(4, h, [(2 * f0, 2 * f1)], (0, f1 - f0))  # pair-product output: f/N rows
    down = Shard(6, f, [(q0, q1)], (0, q1 - q0))
    head = Shard(6, h, [(v0, v1)], (0, v1 - v0))
    return {"qkv": qkv, "o": o, "gate_up": gate_up, "down": down, "head": head}


FULL_KEYS = ("q", "o", "a", "xd", "logits")


def full_sizes(cfg: StackConfig) -> dict[str, int]:
    return {"q": cfg.hidden, "o": cfg.hidden, "a": cfg.ffn, "xd": cfg.hidden, "logits": cfg.vocab}


def push_splits(cfg: StackConfig, world: int, sm_count: int) -> dict[str, int]:
    """Split K per pushed vector (by the vector its matvec writes): 2 where the shard has so few
    16-row bands that half the CTAs would hold one (a CTA's time is its tiles, so two CTAs taking
    half a band's K-tiles each halve it), the rows have two K-tiles or more (more than 16
    super-blocks) and the outputs are plain sums (not the gate/up product); else 1."""
    h, f = cfg.hidden, cfg.ffn
    rows_k = {"q": (h + 2 * cfg.kv, h), "o": (h, h), "xd": (h, f)}
    out = {}
    for key, (rows, k) in rows_k.items():
        bands = -(-(rows // world) // 16)
        out[key] = 2 if world > 1 and 2 * bands <= sm_count and k // QK > 16 else 1
    return out


def push_layout(cfg: StackConfig, splits: dict[str, int] | None = None) -> tuple[dict[str, int], int]:
    """Byte offsets in a rank's exchange region (identical on every rank): the token counter
    ("epoch") in the first 256 bytes, then the tagged full vectors (8 bytes an element: the f32
    value and its tag; a vector written with split K has that many slots of it), each 256-byte
    aligned. Returns (offsets, total bytes)."""
    splits = splits or {}
    off = {"epoch": 0}
    pos = 256
    for k, n in full_sizes(cfg).items():
        off[k] = pos
        pos += (splits.get(k, 1) * n * 8 + 255) // 256 * 256
    return off, pos


def push_tag(cfg: StackConfig, key: str, occurrence: int) -> tuple[int, int]:
    """(mul, add) of the tag of full vector `key`'s occurrence-th write of a token (1-based): the
    tag is (t - 1) * writes_per_token + occurrence in token t, so every write of a vector carries
    a tag no earlier write carried, and no tag is 0 (zeroed memory's)."""
    per_token = 1 if key == "logits" else cfg.layers
    return per_token, occurrence


@dataclass(frozen=True)
class ChainJob:
    """One matvec of a token as a chain job (kq_matvec_chain): what it reads and writes, and the
    counters that order it. Buffer names are full vectors ("x", "q", "o", "a", "xd", "logits",
    read or pushed) or local outputs ("qkv", "o_loc", "a_loc", "x_loc", "l_loc")."""
    name: str
    layer: int
    qtype: int
    rows: int           # this rank's rows of the matrix
    k: int
    x: str              # the full vector it reads
    y: str              # the local buffer that gets every output
    push: str | None    # the full vector its outputs [0, push_rows) go to on every rank (world > 1)
    push_rows: int
    rmsnorm: bool
    pair_scale: float | None
    counter: int        # the counter its CTAs add to (index into the token's counters)
    wait: int | None    # the counter x waits for, or None (the token's input)
    wait_target: int    # what `wait` gains per token
    outputs: int        # outputs on this rank (rows, or rows / 2 for the pair product)


def chain_plan(cfg: StackConfig, rank: int, world: int) -> tuple[list[ChainJob], list[list[int]]]:
    """A token of the stack as chain jobs, and how they group into launches (runs of jobs with
    one type and k, at most 8: per layer q|k|v, o, gate|up in one launch and down in another,
    then the head). Job i adds to counter i: with one rank every output it stores, with N ranks
    the outputs it pushes to every rank's full vector (N * push_rows per token on each rank), and
    the job that reads that vector waits for exactly that count."""
    sh = plan(cfg, rank, world)
    h, f = cfg.hidden, cfg.ffn
    jobs: list[ChainJob] = []

    def add(name, layer, x, y, push, push_rows, rmsnorm=False, pair_scale=None):
        shard = sh[name]
        outputs = shard.rows // 2 if pair_scale is not None else shard.rows
        prev = jobs[-1] if jobs else None
        if prev is None:
            wait, target = None, 0
        else:
            wait = prev.counter
            target = prev.outputs if world == 1 else world * prev.push_rows
        jobs.append(ChainJob(name, layer, shard.qtype, shard.rows, shard.k, x, y,
                             push if world > 1 else None, push_rows if world > 1 else 0, rmsnorm,
                             pair_scale, len(jobs), wait, target, outputs))

    for layer in range(cfg.layers):
        add("qkv", layer, "x" if layer == 0 else "xd", "qkv", "q", h // world, rmsnorm=layer > 0)
        add("o", layer, "q", "o_loc", "o", h // world)
        add("gate_up", layer, "o", "a_loc", "a", f // world, pair_scale=1.0 / math.sqrt(f))
        add("down", layer, "a", "x_loc", "xd", h // world)
    add("head", cfg.layers, "xd" if cfg.layers else "x", "l_loc", "logits", cfg.vocab // world,
        rmsnorm=True)
    launches: list[list[int]] = []
    for i, j in enumerate(jobs):
        cur = launches[-1] if launches else None
        if cur and len(cur) < 8 and (jobs[cur[0]].qtype, jobs[cur[0]].k) == (j.qtype, j.k):
            cur.append(i)
        else:
            launches.append([i])
    return jobs, launches


def chain_layout(cfg: StackConfig, njobs: int) -> tuple[dict[str, int], int]:
    """Byte offsets in a rank's region for chains (identical on every rank): the step counter
    ("epoch") and one u64 counter per job of the token ("counters"), then the full vectors, each
    256-byte aligned. Returns (offsets, total bytes)."""
    off = {"epoch": 0, "counters": 8}
    pos = (8 + 8 * njobs + 255) // 256 * 256
    for k, n in full_sizes(cfg).items():
        off[k] = pos
        pos += (n * 4 + 255) // 256 * 256
    return off, pos


class DecodeStack:
    """One rank's part of a decode stack on a backend. `forward(x)` runs one token."""

    def __init__(self, cfg: StackConfig, backend, rank: int = 0, world: int = 1):
        self.cfg, self.be, self.rank, self.world = cfg, backend, rank, world
        self.shards = plan(cfg, rank, world)
        self.weights = []
        for layer in range(cfg.layers):
            lw = {}
            for name in ("qkv", "o", "gate_up", "down"):
                lw[name] = backend.weights(self.shards[name], cfg.seed, cfg.tensor_id(layer, name))
            self.weights.append(lw)
        self.head = backend.weights(self.shards["head"], cfg.seed, cfg.tensor_id(cfg.layers, "head"))
        h, f = cfg.hidden, cfg.ffn
        sh = self.shards
        full = getattr(backend, "full_vectors", None)
        fv = full(cfg, rank, world) if full else {k: backend.vector(n) for k, n in full_sizes(cfg).items()}
        self.buf = {
            "x": backend.vector(h), "qkv": backend.vector(sh["qkv"].rows), "q": fv["q"],
            "o_loc": backend.vector(sh["o"].rows), "o": fv["o"],
            "a_loc": backend.vector(sh["gate_up"].rows // 2), "a": fv["a"],
            "x_loc": backend.vector(sh["down"].rows), "xd": fv["xd"],
            "l_loc": backend.vector(sh["head"].rows), "logits": fv["logits"],
        }
        self.pos = 0
        if cfg.attention:
            if (cfg.n_heads % world or cfg.n_kv % world or cfg.n_heads % cfg.n_kv
                    or cfg.hidden % cfg.head_dim or cfg.kv % cfg.head_dim):
                raise ValueError("attention needs whole heads on every rank and whole query groups")
            nq = sh["qkv"].gathered[1]  # this rank's query rows = its heads' attention outputs
            self.buf["q_rot"] = backend.vector(nq)
            self.buf["att"] = backend.vector(nq)
            self.caches = [backend.kv_cache(cfg, world) for _ in range(cfg.layers)]
        if world == 1:
            # one rank: each "gathered" vector is the local output itself (q is the first h
            # entries of the q|k|v output, or the attention output), so the gathers vanish
            b = self.buf
            b["q"] = b["att"] if cfg.attention else b["qkv"]
            b["o"], b["a"], b["xd"], b["logits"] = b["o_loc"], b["a_loc"], b["x_loc"], b["l_loc"]

    def launches_per_token(self) -> int:
        """This library's kernels per token: the matvecs (chains: the step counter's advance and
        one launch per run of jobs), plus the closing wait of an exchange between GPUs."""
        if getattr(self.be, "chain", False):
            return 1 + len(self.be.chain_launches) + (1 if self.world > 1 else 0)
        return 4 * self.cfg.layers + 1 + (1 if getattr(self.be, "push", False) else 0)

    def forward(self) -> None:
        """One token: reads buf['x'], writes buf['logits'] (on every rank)."""
        if getattr(self.be, "chain", False):
            self.be.chain_token(self)
            return
        cfg, be, b, sh = self.cfg, self.be, self.buf, self.shards
        begin = getattr(be, "begin_token", None)
        if begin:
            begin()
        x = b["x"]
        if cfg.attention and self.pos >= cfg.max_pos:
            raise ValueError(f"the key/value caches hold {cfg.max_pos} positions")
        for layer, lw in enumerate(self.weights):
            be.matvec(lw["qkv"], sh["qkv"], b["qkv"], x, rmsnorm=layer > 0, eps=cfg.eps,
                      out=("q", sh["qkv"].gathered, layer + 1), src=("xd", layer) if layer > 0 else None)
            if cfg.attention:
                # this rank's heads: rotate, append to the layer's cache, attend; o's input is
                # every rank's attention output
                be.attend(self, layer, self.pos)
                be.gather(b["q"], b["att"], (0, sh["qkv"].gathered[1]))
            else:
                be.gather(b["q"], b["qkv"], sh["qkv"].gathered)
            be.matvec(lw["o"], sh["o"], b["o_loc"], b["q"], out=("o", sh["o"].gathered, layer + 1),
                      src=("q", layer + 1))
            be.gather(b["o"], b["o_loc"], sh["o"].gathered)
            be.matvec(lw["gate_up"], sh["gate_up"], b["a_loc"], b["o"], pair_scale=1.0 / math.sqrt(cfg.ffn),
                      out=("a", sh["gate_up"].gathered, layer + 1), src=("o", layer + 1))
            be.gather(b["a"], b["a_loc"], sh["gate_up"].gathered)
            be.matvec(lw["down"], sh["down"], b["x_loc"], b["a"], out=("xd", sh["down"].gathered, layer + 1),
                      src=("a", layer + 1))
            be.gather(b["xd"], b["x_loc"], sh["down"].gathered)
            x = b["xd"]
        be.matvec(self.head, sh["head"], b["l_loc"], x, rmsnorm=True, eps=cfg.eps,
                  out=("logits", sh["head"].gathered, 1), src=("xd", cfg.layers) if self.cfg.layers else None)
        be.gather(b["logits"], b["l_loc"], sh["head"].gathered)
        end = getattr(be, "end_token", None)
        if end:
            end(self)
        self.pos += 1


# ---------------------------------------------------------------- the CUDA backend (product)

class CudaBackend:
    """libkq.so kernels on one GPU. With world > 1 the exchange after each projection is either
    an NCCL all-gather (torch.distributed), or -- push=True -- done by the matvec itself: its
    epilogue stores its rows into every rank's full vector over CUDA IPC peer mappings and
    counts them there, and the next matvec waits for the count (kq_matvec_push), or -- chain=True
    -- the same inside chains of several matvecs per launch (kq_matvec_chain)."""

    def __init__(self, kernels, stream=None, group=None, world: int = 1, flags: int = 0,
                 push: bool = False, rank: int = 0, chain: bool = False, split_k: bool = False):
        import torch

        import kernite_b200 as kb

        self.kb, self.torch, self.k = kb, torch, kernels
        self.stream = stream
        self.group = group
        self.world = world
        self.rank = rank
        self.flags = flags
        self.chain = chain
        self.split_k = split_k
        self.push = push and world > 1 and not chain
        self.launches = 0
        self.region = None
        self.peers: list[int] = []

    # ---------------------------------------------------------------- push exchange set-up
    def _map_region(self, nbytes: int, rank: int, world: int) -> None:
        """This rank's exchange region (zeroed, IPC-shareable) and every peer's, mapped."""
        import torch.distributed as dist

        ptr, handle = self.k.peer_alloc(nbytes)
        self.region = ptr
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=self.group)
        self.peers = [ptr if p == rank else self.k.peer_open(handles[p]) for p in range(world)]

    def full_vectors(self, cfg: StackConfig, rank: int, world: int):
        torch, kb = self.torch, self.kb
        if self.chain:
            return self._chain_vectors(cfg, rank, world)
        if not self.push:
            return {k: self.vector(n) for k, n in full_sizes(cfg).items()}
        # the exchange's full vectors are tagged, in the region every rank maps; the host-side
        # vectors are plain ones (the logits unpacked into buf['logits'] at the end of a token)
        self.cfg = cfg
        # split K for short shards (push_splits) measured no faster on a B200 at 8-way shards
        # (62.1 vs 62.4 us a 70B layer: the readers' two-slot loads cost what the halved tiles
        # save), so the stack pushes unsplit; the library keeps the option (KqPushDesc.ksplit)
        self.ksplit = push_splits(cfg, world, self.k.sm_count) if self.split_k else {}
        self.off, nbytes = push_layout(cfg, self.ksplit)
        self._map_region(nbytes, rank, world)
        self.epoch = torch.as_tensor(kb.DeviceArray(self.region + self.off["epoch"], 1, "<i8"), device="cuda")
        return {k: self.vector(n) for k, n in full_sizes(cfg).items()}

    # ---------------------------------------------------------------- chains
    def _chain_vectors(self, cfg: StackConfig, rank: int, world: int):
        """Chains: the token's jobs, the step counter and job counters, and the full vectors (in
        the exchange region every rank maps when world > 1)."""
        torch, kb = self.torch, self.kb
        self.cfg = cfg
        self.chain_jobs, self.chain_launches = chain_plan(cfg, rank, world)
        off, nbytes = chain_layout(cfg, len(self.chain_jobs))
        self.coff = off
        if world == 1:
            self._counter_mem = torch.zeros(1 + len(self.chain_jobs), dtype=torch.int64, device="cuda")
            base = self._counter_mem.data_ptr()
            self.epoch_addr, self.counter_base = base, base + 8
            return {k: self.vector(n) for k, n in full_sizes(cfg).items()}
        self._map_region(nbytes, rank, world)
        self.epoch_addr = self.region + off["epoch"]
        self.counter_base = self.region + off["counters"]
        view = lambda o, n: torch.as_tensor(kb.DeviceArray(self.region + o, n), device="cuda")
        return {k: view(off[k], n) for k, n in full_sizes(cfg).items()}

    def build_chains(self, stack: "DecodeStack") -> None:
        """The kq_chain_job arrays of every launch of a token (addresses fixed from here on)."""
        kb = self.kb
        b = stack.buf
        self.chain_arrays = []
        for launch in self.chain_launches:
            arr = (kb.KqChainJob * len(launch))()
            for slot, i in enumerate(launch):
                j = self.chain_jobs[i]
                if j.layer < stack.cfg.layers:
                    W = stack.weights[j.layer][j.name]
                else:
                    W = stack.head
                d = arr[slot]
                d.mv = kb.KqMatvecDesc(
                    type={4: kb.TYPE_Q4_K, 6: kb.TYPE_Q6_K}[j.qtype], rows=j.rows, k=j.k, batch=1,
                    y=b[j.y].data_ptr(), w=W.data_ptr(), x=b[j.x].data_ptr(), ldx=0, ldy=0,
                    prologue=kb.PROLOGUE_RMSNORM if j.rmsnorm else kb.PROLOGUE_NONE,
                    epilogue=kb.EPILOGUE_PAIR_PRODUCT if j.pair_scale is not None else kb.EPILOGUE_NONE,
                    eps=stack.cfg.eps, pair_scale=j.pair_scale if j.pair_scale is not None else 1.0,
                    flags=kb.FLAG_WEIGHTS_STATIC | self.flags, reserved=0)
                if j.wait is not None:
                    d.wait_counter = self.counter_base + 8 * j.wait
                    d.wait_target = j.wait_target
                if self.world == 1:
                    d.npush = 0
                    d.counter[0] = self.counter_base + 8 * j.counter
                else:
                    d.npush = self.world
                    d.push_rows = j.push_rows
                    for p, base in enumerate(self.peers):
                        d.push_y[p] = base + self.coff[j.push] + 4 * self.rank * j.push_rows
                        d.counter[p] = base + self.coff["counters"] + 8 * j.counter
            self.chain_arrays.append(arr)

    def chain_token(self, stack: "DecodeStack") -> None:
        """One token as chains: advance the step counter, launch every run of jobs, and (world
        > 1) wait until every rank's logits have arrived."""
        if not hasattr(self, "chain_arrays"):
            self.build_chains(stack)
        self.k.epoch_advance(self.epoch_addr, stream=self.stream)
        for arr in self.chain_arrays:
            self.k.matvec_chain(arr, self.epoch_addr, stream=self.stream)
        self.launches += 1 + len(self.chain_arrays)
        if self.world > 1:
            head = self.chain_jobs[-1]
            n = self.world * head.push_rows
            self.k.wait_counter(self.counter_base + 8 * head.counter, self.epoch_addr, n, n,
                                stream=self.stream)
            self.launches += 1

    def begin_token(self) -> None:
        if self.push:
            with self.torch.cuda.stream(self.stream) if self.stream is not None else _null():
                self.epoch.add_(1)

    def end_token(self, stack: "DecodeStack" = None) -> None:
        # the logits are the one pushed vector no later launch reads: wait for every rank's rows
        # and unpack them into the plain logits
        if self.push:
            self.k.tagged_unpack(stack.buf["logits"], self.region + self.off["logits"], self.cfg.vocab,
                                 self.region + self.off["epoch"], *push_tag(self.cfg, "logits", 1),
                                 stream=self.stream)
            self.launches += 1

    def close(self) -> None:
        """Unmaps the peers' regions and frees this rank's, once every rank is done with them
        (a collective step: all ranks call it)."""
        self.torch.cuda.synchronize()
        if self.peers:
            import torch.distributed as dist

            dist.barrier(group=self.group)
        for p, ptr in enumerate(self.peers):
            if p != self.rank:
                self.k.peer_close(ptr)
        if self.region:
            self.k.peer_free(self.region)
        self.peers, self.region = [], None

    # ---------------------------------------------------------------- weights and vectors
    def weights(self, shard: Shard, seed: int, tensor: int):
        torch, kb = self.torch, self.kb
        W = torch.empty(shard.nbytes, dtype=torch.uint8, device="cuda")
        key = kb.stream_key(seed, tensor)
        nb = shard.k // QK
        bb = BLOCK_BYTES[shard.qtype]
        off = 0
        for r0, r1 in shard.runs:
            n = (r1 - r0) * nb
            self.k.fill(shard.qtype, W.data_ptr() + off, r0 * nb, n, key, stream=self.stream)
            off += n * bb
        return W

    def vector(self, n: int):
        return self.torch.zeros(n, dtype=self.torch.float32, device="cuda")

    def kv_cache(self, cfg: StackConfig, world: int):
        """One layer's f16 key and value caches for this rank's key/value heads."""
        n = cfg.max_pos * (cfg.n_kv // world) * cfg.head_dim
        torch = self.torch
        return (torch.zeros(n, dtype=torch.float16, device="cuda"),
                torch.zeros(n, dtype=torch.float16, device="cuda"))

    def attend(self, stack: "DecodeStack", layer: int, pos: int) -> None:
        """This rank's heads of one layer's attention at position pos: q and k rotated, k and v
        appended to the layer's cache, buf['att'] = attention over positions 0..pos."""
        cfg, b, w = stack.cfg, stack.buf, self.world
        nh, nkv, d = cfg.n_heads // w, cfg.n_kv // w, cfg.head_dim
        kc, vc = stack.caches[layer]
        if not hasattr(self, "_att_ws"):
            nbytes = self.k.attention_workspace(nh, nkv, d, cfg.max_pos)
            self._att_ws = self.torch.empty(nbytes // 4 + 4, dtype=self.torch.float32, device="cuda")
        self.k.rope_append(b["qkv"], b["q_rot"], kc, vc, nh, nkv, d, pos, cfg.rope_base, stream=self.stream)
        self.k.attention(b["att"], b["q_rot"], kc, vc, nh, nkv, d, pos + 1, self._att_ws,
                         self._att_ws.numel() * 4, stream=self.stream)
        self.launches += 3

    def matvec(self, W, shard: Shard, y, x, rmsnorm: bool = False, eps: float = 0.0,
               pair_scale: float | None = None, out=None, src=None) -> None:
        kb = self.kb
        kw = dict(prologue=kb.PROLOGUE_RMSNORM if rmsnorm else kb.PROLOGUE_NONE, eps=eps,
                  epilogue=kb.EPILOGUE_PAIR_PRODUCT if pair_scale is not None else kb.EPILOGUE_NONE,
                  pair_scale=pair_scale if pair_scale is not None else 1.0,
                  flags=kb.FLAG_WEIGHTS_STATIC | self.flags, stream=self.stream)
        if self.push and out is not None:
            key, (a, b), occ_out = out
            d = kb.KqPushDesc()
            d.npush = self.world
            d.push_rows = b - a
            d.flags = kb.PUSH_TAGGED
            d.epoch = self.region + self.off["epoch"]
            d.push_mul, d.push_add = push_tag(self.cfg, key, occ_out)
            d.ksplit = self.ksplit.get(key, 1) if pair_scale is None else 1
            for p, base in enumerate(self.peers):
                d.y[p] = base + self.off[key] + 8 * self.rank * (b - a)
            if src is not None:
                # x is this rank's tagged copy of the full vector (the sum of its split-K slots)
                skey, occ = src
                d.flags |= kb.PUSH_TAGGED_X
                d.wait_mul, d.wait_add = push_tag(self.cfg, skey, occ)
                d.x_slots = self.ksplit.get(skey, 1)
                x = self.region + self.off[skey]
            self.k.matvec_push(shard.qtype, y, W, x, shard.rows, shard.k, d, **kw)
        else:
            self.k.matvec(shard.qtype, y, W, x, shard.rows, shard.k, 1, **kw)
        self.launches += 1

    def gather(self, out, loc, part: tuple[int, int]) -> None:
        if self.world == 1 or self.push:
            return  # aliased (one rank) or pushed by the matvec itself
        import torch.distributed as dist

        a, b = part
        dist.all_gather_into_tensor(out, loc[a:b], group=self.group)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def make_cuda_stack(cfg: StackConfig, kernels, rank: int = 0, world: int = 1, group=None,
                    stream=None, flags: int = 0, push: bool = False, chain: bool = False,
                    split_k: bool = False) -> DecodeStack:
    if cfg.attention and (push or chain):
        raise ValueError("a stack with attention runs one launch per projection (NCCL or one rank)")
    """One rank's stack on libkq.so. The exchange between ranks (and the launches): NCCL
    all-gathers after one matvec launch per projection (default), the matvec's own push to peer
    memory (push=True, the warp-MMA kernel's push variant), or chains (chain=True: up to
    three projections per launch, outputs pushed to peer memory and ordered by counters)."""
    return DecodeStack(cfg, CudaBackend(kernels, stream=stream, group=group, world=world, flags=flags,
                                        push=push, rank=rank, chain=chain, split_k=split_k), rank, world)


# ---------------------------------------------------------------- reference (for tests)

def _reference_attend(cfg: StackConfig, layer: int, qkv, cache: dict):
    """One layer's attention step of the reference: rotate q and k at the next position, append
    k and v (rounded to f16, as the GPU's caches hold them), attend over every position so far."""
    import numpy as np

    import oracle

    nh, nkv, d = cfg.n_heads, cfg.n_kv, cfg.head_dim
    pos = cache.setdefault("pos", 0)
    q, k, v = oracle.rope_ref(qkv, nh, nkv, d, pos, cfg.rope_base)
    K, V = cache.setdefault(layer, ([], []))
    K.append(k.astype(np.float32).astype(np.float16))
    V.append(v.astype(np.float32).astype(np.float16))
    att, _ = oracle.attention_ref(q.astype(np.float32), np.stack(K), np.stack(V), nh, nkv, d, pos + 1)
    return att.reshape(-1)


def reference_logits(cfg: StackConfig, x, layers: int | None = None, with_bound: bool = False,
                     cache: dict | None = None):
    """The unsharded stack on the CPU oracle, in f64 from the f32-dequantised weights; with
    `with_bound` also sum_k |w_head[r, k] x_k| per logit (x the normalised head input), the scale
    of the 1e-3 tolerance. With attention, `cache` carries the key/value caches and the position
    from one call (token) to the next. Test and bench-check infrastructure only."""
    if cache is None:
        cache = {}
    import numpy as np

    import oracle

    def weights(name, layer, qtype, rows, k):
        return oracle.fill(qtype, oracle.stream_key(cfg.seed, cfg.tensor_id(layer, name)), 0,
                           rows * k // QK)

    def mv(qtype, W, v, rows, k, bound=False):
        y, b = oracle.matvec_ref(qtype, W, np.asarray(v, dtype=np.float32)[None, :], k, 0, rows)
        return (y[0], b[0]) if bound else y[0]

    def norm(v):
        v = np.asarray(v, dtype=np.float64)
        return v / np.sqrt(np.mean(v * v) + cfg.eps)

    h, f, kv = cfg.hidden, cfg.ffn, cfg.kv
    x = np.asarray(x, dtype=np.float64)
    nl = cfg.layers if layers is None else layers
    for layer in range(nl):
        xin = norm(x) if layer > 0 else x
        qkv = mv(4, weights("qkv", layer, 4, h + 2 * kv, h), xin, h + 2 * kv, h)
        q = qkv[:h]
        if cfg.attention:
            q = _reference_attend(cfg, layer, qkv, cache)
        o = mv(4, weights("o", layer, 4, h, h), q, h, h)
        gu = mv(4, weights("gate_up", layer, 4, 2 * f, h), o, 2 * f, h)
        a = gu[0::2] * gu[1::2] / math.sqrt(f)
        x = mv(6, weights("down", layer, 6, h, f), a, h, f)
    head = oracle.fill(6, oracle.stream_key(cfg.seed, cfg.tensor_id(cfg.layers, "head")), 0,
                       cfg.vocab * h // QK)
    logits, bound = mv(6, head, norm(x), cfg.vocab, h, bound=True)
    if cfg.attention:
        cache["pos"] += 1
    return (logits, bound) if with_bound else logits
