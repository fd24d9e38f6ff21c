"""Seeded synthetic workloads with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; these generators stand in for it with the
shapes, sizes and value distributions the configurations name:

* C1  Qwen2.5-0.5B decode:  Hq 14, Hkv 2, d 64, bs 16, B 4, ctx ~ U[33, 512], f32 ~ N(0,1)/8,
      block tables a seeded permutation of a 256-block pool.
* C2  Llama-3-8B decode:    Hq 32, Hkv 8, d 128, bs 16, B 64, ctx ~ U[512, 4096], bf16 ~ N(0,1),
      32 layers, shuffled non-contiguous block tables.
* C3  varlen prefill:       Llama-3-8B heads, 16 sequences, L ~ U[128, 2048] in groups of 4 that
      share a prefix of 0-50% of the group's shortest length (multiple of 16, same physical
      blocks in all 4 tables); only suffix tokens are queried; their K/V go through
      reshape_and_cache.
* C4  long context decode:  B 16, ctx ~ U[16384, 32768], Llama-3-8B heads.
* C5  Qwen2-7B mixed step:  Hq 28, Hkv 4, d 128, ctx ~ LogNormal(ln 1024, 0.8) capped at 8192.

Lengths and permutations come from numpy's PCG64 seeded with ``seed``; tensor contents from a
torch generator seeded with the same value on the target device.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Heads:
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int = 16

    @property
    def n_rep(self) -> int:
        return self.num_heads // self.num_kv_heads


QWEN05 = Heads(14, 2, 64)
LLAMA8B = Heads(32, 8, 128)
QWEN7B = Heads(28, 4, 128)


@dataclass
class DecodeBatch:
    heads: Heads
    dtype: torch.dtype
    q: torch.Tensor                    # [B, Hq, d]
    k_caches: list                     # per layer [num_blocks, Hkv, bs, d]
    v_caches: list
    block_tables: torch.Tensor         # int32 [B, max_blocks]
    context_lens: torch.Tensor         # int32 [B]
    ctx_host: np.ndarray
    max_context_len: int
    num_blocks: int

    @property
    def num_seqs(self) -> int:
        return int(self.q.shape[0])

    def kv_bytes_per_layer(self) -> int:
        """Algorithmic HBM bytes one decode launch must read: K and V of every live token."""
        h = self.heads
        es = torch.tensor([], dtype=self.dtype).element_size()
        return int(self.ctx_host.sum()) * h.num_kv_heads * h.head_dim * 2 * es

    def io_bytes_per_layer(self) -> int:
        """Everything else a launch touches: q, out, block-table entries, context lengths."""
        h = self.heads
        es = torch.tensor([], dtype=self.dtype).element_size()
        pages = int(((self.ctx_host + h.block_size - 1) // h.block_size).sum())
        return 2 * self.num_seqs * h.num_heads * h.head_dim * es + 4 * pages + 4 * self.num_seqs


def _randn(shape, dtype, device, gen, scale=1.0):
    t = torch.randn(shape, dtype=torch.float32, device=device, generator=gen)
    if scale != 1.0:
        t.mul_(scale)
    return t.to(dtype)


def make_decode(heads: Heads, ctx: np.ndarray, dtype: torch.dtype, device, seed: int,
                num_layers: int = 1, value_scale: float = 1.0, pool_blocks: int | None = None,
                fill: bool = True) -> DecodeBatch:
    """A decode batch whose sequences own disjoint, randomly placed blocks of a shared pool."""
    rng = np.random.default_rng(seed)
    bs = heads.block_size
    ctx = np.asarray(ctx, dtype=np.int64)
    pages = (ctx + bs - 1) // bs
    need = int(pages.sum())
    nb = max(need, pool_blocks or 0)
    perm = rng.permutation(nb).astype(np.int32)
    max_blocks = int(pages.max())
    bt = np.zeros((len(ctx), max_blocks), dtype=np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n]
        o += n
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shape = (nb, heads.num_kv_heads, bs, heads.head_dim)
    kc, vc = [], []
    for _ in range(num_layers):
        if fill:
            kc.append(_randn(shape, dtype, device, gen, value_scale))
            vc.append(_randn(shape, dtype, device, gen, value_scale))
        else:
            kc.append(torch.empty(shape, dtype=dtype, device=device))
            vc.append(torch.empty(shape, dtype=dtype, device=device))
    q = _randn((len(ctx), heads.num_heads, heads.head_dim), dtype, device, gen, value_scale)
    return DecodeBatch(heads, dtype, q, kc, vc, torch.from_numpy(bt).to(device),
                       torch.from_numpy(ctx.astype(np.int32)).to(device), ctx.astype(np.int32),
                       int(ctx.max()), nb)


def c1_contexts(seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(33, 513, size=4)


def c2_contexts(seed: int, batch: int = 64) -> np.ndarray:
    return np.random.default_rng(seed).integers(512, 4097, size=batch)


def c4_contexts(seed: int, batch: int = 16) -> np.ndarray:
    return np.random.default_rng(seed).integers(16384, 32769, size=batch)


def c5_contexts(seed: int, n: int = 512) -> np.ndarray:
    x = np.random.default_rng(seed).lognormal(np.log(1024.0), 0.8, size=n)
    return np.clip(np.round(x), 1, 8192).astype(np.int64)


def make_c1(device, seed: int = 1) -> DecodeBatch:
    """C1 with the pool fixed at 256 blocks and the tables a seeded permutation of it."""
    return make_decode(QWEN05, c1_contexts(seed), torch.float32, device, seed,
                       value_scale=1.0 / 8.0, pool_blocks=256)


@dataclass
class PrefillBatch:
    heads: Heads
    dtype: torch.dtype
    q: torch.Tensor                 # [Tq, Hq, d] suffix queries, packed
    key: torch.Tensor               # [Tq, Hkv, d] suffix keys (written by reshape_and_cache)
    value: torch.Tensor
    k_caches: list
    v_caches: list
    cu_seqlens_q: torch.Tensor      # int32 [S+1]
    context_lens: torch.Tensor      # int32 [S] prefix + suffix
    block_tables: torch.Tensor      # int32 [S, max_blocks]
    slot_mapping: torch.Tensor      # int32 [Tq]
    lens: np.ndarray                # total length per sequence
    prefix: np.ndarray              # cached prefix length per sequence
    max_seqlen_q: int
    max_context_len: int
    num_blocks: int

    def flops(self) -> int:
        """Causal suffix-only FLOPs: sum 4*Hq*d*(S*P + S(S+1)/2) (masked work not counted)."""
        h = self.heads
        S = (self.lens - self.prefix).astype(np.int64)
        P = self.prefix.astype(np.int64)
        return int((4 * h.num_heads * h.head_dim * (S * P + S * (S + 1) // 2)).sum())


def make_c3(device, seed: int = 3, dtype=torch.bfloat16, num_layers: int = 1,
            heads: Heads = LLAMA8B, num_seqs: int = 16, group: int = 4, lo: int = 128,
            hi: int = 2048, max_prefix_frac: float = 0.5) -> PrefillBatch:
    """C3: groups of `group` sequences share a cached prefix; suffixes are new tokens."""
    rng = np.random.default_rng(seed)
    bs = heads.block_size
    lens = rng.integers(lo, hi + 1, size=num_seqs)
    prefix = np.zeros(num_seqs, dtype=np.int64)
    for g0 in range(0, num_seqs, group):
        f = rng.uniform(0.0, max_prefix_frac)
        p = int(f * lens[g0:g0 + group].min()) // bs * bs
        prefix[g0:g0 + group] = p
    # Physical blocks: one shared run per group for the prefix, private blocks for the rest.
    n_shared = [int(prefix[g0]) // bs for g0 in range(0, num_seqs, group)]
    n_private = [int((lens[i] - prefix[i] + bs - 1) // bs) for i in range(num_seqs)]
    total = sum(n_shared) + sum(n_private)
    perm = rng.permutation(total).astype(np.int32)
    max_blocks = int(((lens + bs - 1) // bs).max())
    bt = np.zeros((num_seqs, max_blocks), dtype=np.int32)
    o = 0
    for gi, g0 in enumerate(range(0, num_seqs, group)):
        shared = perm[o:o + n_shared[gi]]
        o += n_shared[gi]
        for i in range(g0, min(g0 + group, num_seqs)):
            bt[i, :len(shared)] = shared
            bt[i, len(shared):len(shared) + n_private[i]] = perm[o:o + n_private[i]]
            o += n_private[i]
    suffix = lens - prefix
    cu = np.concatenate([[0], np.cumsum(suffix)]).astype(np.int32)
    slots = []
    for i in range(num_seqs):
        for pos in range(int(prefix[i]), int(lens[i])):
            slots.append(int(bt[i, pos // bs]) * bs + pos % bs)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shape = (total, heads.num_kv_heads, bs, heads.head_dim)
    kc = [_randn(shape, dtype, device, gen) for _ in range(num_layers)]
    vc = [_randn(shape, dtype, device, gen) for _ in range(num_layers)]
    tq = int(cu[-1])
    q = _randn((tq, heads.num_heads, heads.head_dim), dtype, device, gen)
    key = _randn((tq, heads.num_kv_heads, heads.head_dim), dtype, device, gen)
    value = _randn((tq, heads.num_kv_heads, heads.head_dim), dtype, device, gen)
    return PrefillBatch(heads, dtype, q, key, value, kc, vc,
                        torch.from_numpy(cu).to(device),
                        torch.from_numpy(lens.astype(np.int32)).to(device),
                        torch.from_numpy(bt).to(device),
                        torch.tensor(slots, dtype=torch.int32, device=device),
                        lens.astype(np.int64), prefix, int(suffix.max()), int(lens.max()), total)


def make_prefill(heads: Heads, lens, prefix, dtype: torch.dtype, device, seed: int,
                 num_layers: int = 1) -> PrefillBatch:
    """A packed prefill batch: sequence i holds lens[i] tokens, the first prefix[i] of them
    already cached; every sequence owns private, randomly placed blocks of one pool. Pools,
    queries and new K/V are seeded N(0,1)."""
    rng = np.random.default_rng(seed)
    bs = heads.block_size
    lens = np.asarray(lens, dtype=np.int64)
    prefix = np.asarray(prefix, dtype=np.int64)
    pages = (lens + bs - 1) // bs
    total = max(1, int(pages.sum()))
    perm = rng.permutation(total).astype(np.int32)
    max_blocks = max(1, int(pages.max()) if len(lens) else 1)
    bt = np.zeros((len(lens), max_blocks), dtype=np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n]
        o += int(n)
    suffix = lens - prefix
    cu = np.concatenate([[0], np.cumsum(suffix)]).astype(np.int32)
    slots = np.concatenate([bt[i, np.arange(prefix[i], lens[i]) // bs] * bs +
                            np.arange(prefix[i], lens[i]) % bs for i in range(len(lens))]
                           ) if len(lens) else np.zeros(0, np.int64)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    make = lambda shape: _randn(shape, dtype, device, gen)  # noqa: E731
    shape = (total, heads.num_kv_heads, bs, heads.head_dim)
    kc = [make(shape) for _ in range(num_layers)]
    vc = [make(shape) for _ in range(num_layers)]
    tq = int(cu[-1])
    q = make((tq, heads.num_heads, heads.head_dim))
    key = make((tq, heads.num_kv_heads, heads.head_dim))
    value = make((tq, heads.num_kv_heads, heads.head_dim))
    return PrefillBatch(heads, dtype, q, key, value, kc, vc,
                        torch.from_numpy(cu).to(device),
                        torch.from_numpy(lens.astype(np.int32)).to(device),
                        torch.from_numpy(bt).to(device),
                        torch.from_numpy(slots.astype(np.int32)).to(device),
                        lens, prefix, int(suffix.max()) if len(lens) else 0,
                        int(lens.max()) if len(lens) else 0, total)


# Per-unit times of the C5 step on one B200, fitted to a measured 8-rank step (Qwen2-7B heads):
# a decode sequence costs its context length x _C5_DECODE_S_PER_TOKEN per layer; a prompt costs
# its prefill work units x _C5_PREFILL_S_PER_UNIT, where a unit is one 128-token KV tile of one
# work item (a 2 x TQ-token chunk and one KV head) and each item adds _C5_ITEM_UNITS units for
# its epilogue. Short prompts are dearer than their FLOPs because of that per-item cost.
_C5_DECODE_S_PER_TOKEN = 5.5e-10
_C5_PREFILL_S_PER_UNIT = 1.51e-8
_C5_ITEM_UNITS = 3


def prefill_units(S: int, heads: Heads, prefix: int = 0, tile: int = 128) -> int:
    """Work units of the tcgen05 prefill kernel for one prompt of S new tokens after `prefix`
    cached ones: per (chunk of 2 * (128 // n_rep) tokens, KV head) item, its KV tiles plus the
    epilogue's share."""
    chunk = 2 * (128 // heads.n_rep)
    units = 0
    for t0 in range(0, S, chunk):
        kv_end = prefix + min(t0 + chunk, S)
        units += -(-kv_end // tile) + _C5_ITEM_UNITS
    return units * heads.num_kv_heads


def c5_plan(seed: int, n: int = 512, prefill_frac: float = 0.1):
    """C5 mixed serving step (Qwen2-7B heads): 512 sequences with ctx ~ LogNormal(ln 1024, 0.8)
    capped at 8192; a prefill_frac share are new prompts of L ~ U[256, 2048] (no cached prefix),
    the rest decode one token. Returns (ctx, is_prefill, prefill_len, cost) where cost is the
    estimated time per layer of each sequence on one GPU (decode: per context token; prefill: per
    kernel work unit, see prefill_units), for partitioning across GPUs."""
    rng = np.random.default_rng(seed + 55)
    ctx = c5_contexts(seed, n)
    is_pf = rng.random(n) < prefill_frac
    pf_len = rng.integers(256, 2049, size=n)
    dec_cost = ctx * _C5_DECODE_S_PER_TOKEN
    pf_cost = np.array([prefill_units(int(x), QWEN7B) * _C5_PREFILL_S_PER_UNIT for x in pf_len])
    return ctx, is_pf, pf_len, np.where(is_pf, pf_cost, dec_cost)


def mixed_partition(costs, is_prefill, parts: int, overlap: float = 0.5) -> list[list[int]]:
    """Sequence sharding for a step whose decode and prefill sub-batches run on two streams of
    each GPU: a GPU with prefill time P and decode time D is estimated at max(P, D) + overlap *
    min(P, D). Prompts are placed first (longest-first, the larger and coarser work), then each
    decode sequence, longest first, goes where that estimate grows least.

    The estimate is a balancing model, not the measured overlap: on B200 the C5 shares' two
    streams overlap by only 4-8 us per layer (the persistent prefill kernel holds every SM while
    it runs), while the per-token decode cost in c5_plan is above the measured rate by a similar
    margin; with overlap 0.5 the eight measured N=8 shares land within 3 % of each other."""
    costs = np.asarray(costs, dtype=np.float64)
    is_prefill = np.asarray(is_prefill, dtype=bool)
    pf = np.flatnonzero(is_prefill)
    bins = [[int(pf[j]) for j in b] for b in lpt_partition(costs[pf], parts)]
    P = [float(costs[b].sum()) for b in bins]
    D = [0.0] * parts
    for i in np.flatnonzero(~is_prefill)[np.argsort(-costs[~is_prefill], kind="stable")]:
        est = [max(P[r], D[r] + costs[i]) + overlap * min(P[r], D[r] + costs[i]) for r in range(parts)]
        r = int(np.argmin(est))
        bins[r].append(int(i))
        D[r] += float(costs[i])
    return [sorted(b) for b in bins]


def lpt_partition(costs, parts: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of items to `parts` bins (sequence sharding)."""
    order = np.argsort(-np.asarray(costs, dtype=np.float64), kind="stable")
    loads = [0.0] * parts
    bins: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        j = int(np.argmin(loads))
        bins[j].append(int(i))
        loads[j] += float(costs[i])
    return [sorted(b) for b in bins]


@dataclass
class MixedStep:
    """One C5 serving step on one GPU: the decode sequences (one new token each, written and
    attended in one fa_paged_decode_append launch per layer) on the caller's stream and the new
    prompts (fa_reshape_and_cache of their K/V, then fa_paged_prefill, per layer) on a side
    stream, forked and joined inside ``run``. The two sub-batches share no data through any
    layer, so decode CTAs fill the SMs the persistent prefill kernel leaves idle in its tail and
    the other way round. Every layer writes the same output buffers (``dout``, ``pout``)."""
    heads: Heads
    num_layers: int
    dec: DecodeBatch | None
    dk: torch.Tensor | None          # [B, Hkv, d] the decode sequences' new K and V
    dv: torch.Tensor | None
    dout: torch.Tensor | None        # [B, Hq, d]
    pf: PrefillBatch | None
    pout: torch.Tensor | None        # [Tq, Hq, d]
    ws_dec: object = None
    ws_pf: object = None
    side: object = None
    score_flow: int = 0              # FA_SCORES_F32 or FA_SCORES_REFERENCE

    def run_decode(self):
        from . import ops
        h, b = self.heads, self.dec
        scale = 1.0 / float(np.sqrt(h.head_dim))
        for l in range(self.num_layers):
            ops.paged_decode_append(b.q, b.k_caches[l], b.v_caches[l], self.dk, self.dv,
                                    b.block_tables, b.context_lens, h.n_rep, scale,
                                    b.max_context_len, self.ws_dec, out=self.dout,
                                    score_flow=self.score_flow)

    def run_prefill(self):
        from . import ops
        h, b = self.heads, self.pf
        scale = 1.0 / float(np.sqrt(h.head_dim))
        for l in range(self.num_layers):
            ops.reshape_and_cache(b.k_caches[l], b.v_caches[l], b.key, b.value, b.slot_mapping)
            ops.paged_prefill(b.q, b.k_caches[l], b.v_caches[l], b.cu_seqlens_q, b.context_lens,
                              b.block_tables, h.n_rep, scale, b.max_seqlen_q, b.max_context_len,
                              self.ws_pf, out=self.pout, score_flow=self.score_flow)

    def run(self):
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        if self.dec is not None:
            self.run_decode()
        if self.pf is not None:
            with torch.cuda.stream(self.side):
                self.run_prefill()
        main.wait_stream(self.side)


def make_mixed_step(heads: Heads, dec_ctx, pf_len, dtype: torch.dtype, device, seed: int,
                    num_layers: int) -> MixedStep:
    """Seeded N(0,1) pools (only the blocks the tables reference exist), queries and new K/V for
    a mixed step: decode sequences with contexts `dec_ctx` (the new token included) and new
    prompts of lengths `pf_len` with no cached prefix."""
    from . import ops
    dec_ctx = np.asarray(dec_ctx, dtype=np.int64)
    pf_len = np.asarray(pf_len, dtype=np.int64)
    dec = dk = dv = dout = pf = pout = None
    ws_dec = ops.Workspace(device)
    if len(dec_ctx):
        dec = make_decode(heads, dec_ctx, dtype, device, seed, num_layers=num_layers)
        g = torch.Generator(device=device).manual_seed(seed + 11)
        B = dec.num_seqs
        dk = _randn((B, heads.num_kv_heads, heads.head_dim), dtype, device, g)
        dv = _randn((B, heads.num_kv_heads, heads.head_dim), dtype, device, g)
        dout = torch.empty_like(dec.q)
        ws_dec.get(ops.workspace_size(B, heads.num_heads, heads.num_kv_heads, heads.head_dim,
                                      dec.max_context_len, 1))
    if len(pf_len):
        pf = make_prefill(heads, pf_len, np.zeros(len(pf_len), np.int64), dtype, device,
                          seed + 100, num_layers=num_layers)
        pout = torch.empty_like(pf.q)
    return MixedStep(heads, num_layers, dec, dk, dv, dout, pf, pout, ws_dec, ops.Workspace(device),
                     torch.cuda.Stream(device=device))


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> numpy (bf16/f16 as uint16 bit patterns, like the oracle expects)."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


ORACLE_DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
