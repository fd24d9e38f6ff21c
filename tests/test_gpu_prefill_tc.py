"""The tcgen05 varlen prefill kernel (bf16/f16, head_dim 128, block_size 16) against the oracle
(src/backend/cpu.rs:57-112), max-abs 2e-2, across GQA ratios, chunk boundaries, empty and
one-token sequences, long cached prefixes and the full C3 configuration."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import _lib, ops
from flour_b200.workloads import LLAMA8B, QWEN7B, Heads, PrefillBatch, make_c3

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu
TOL = 2e-2


def build(device, heads, lens, prefix, seed, dtype=torch.bfloat16):
    """Explicit per-sequence (length, prefix) batch; prefix blocks private per sequence."""
    rng = np.random.default_rng(seed)
    bs = heads.block_size
    lens = np.asarray(lens, dtype=np.int64)
    prefix = np.asarray(prefix, dtype=np.int64)
    pages = (lens + bs - 1) // bs
    total = int(pages.sum()) + 3
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(lens), max(1, int(pages.max()))), dtype=np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n]
        o += n
    suffix = lens - prefix
    cu = np.concatenate([[0], np.cumsum(suffix)]).astype(np.int32)
    slots = [int(bt[i, pos // bs]) * bs + pos % bs for i in range(len(lens))
             for pos in range(int(prefix[i]), int(lens[i]))]
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (total, heads.num_kv_heads, bs, heads.head_dim)
    kc = torch.randn(shape, device=device, generator=g).to(dtype)
    vc = torch.randn(shape, device=device, generator=g).to(dtype)
    tq = int(cu[-1])
    q = torch.randn((tq, heads.num_heads, heads.head_dim), device=device, generator=g).to(dtype)
    key = torch.randn((tq, heads.num_kv_heads, heads.head_dim), device=device, generator=g).to(dtype)
    val = torch.randn((tq, heads.num_kv_heads, heads.head_dim), device=device, generator=g).to(dtype)
    return PrefillBatch(heads, dtype, q, key, val, [kc], [vc], torch.from_numpy(cu).to(device),
                        torch.from_numpy(lens.astype(np.int32)).to(device),
                        torch.from_numpy(bt).to(device),
                        torch.tensor(slots, dtype=torch.int32, device=device), lens, prefix,
                        int(suffix.max()), int(lens.max()), total)


def run_and_check(b, tol=TOL, flows=(_lib.FA_SCORES_F32,)):
    """Write the suffix K/V, run the prefill in each score flow and compare with the oracle in
    the matching mode (FA_SCORES_F32 <-> score_mode 0, f32 scores; FA_SCORES_REFERENCE <->
    score_mode 1, the reference's bf16 dtype flow of cpu.rs:84-85). Returns the last output."""
    h = b.heads
    scale = 1 / math.sqrt(h.head_dim)
    ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    for flow in flows:
        out = ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q,
                                b.context_lens, b.block_tables, h.n_rep, scale, b.max_seqlen_q,
                                b.max_context_len, ops.Workspace(b.q.device), score_flow=flow)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        want = oracle_attention(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                                b.block_tables, h.n_rep, scale, score_mode=flow)
        err = max_abs(f32(out), want)
        assert err <= tol, f"score flow {flow}: max-abs {err}"
    return out


BOTH = (_lib.FA_SCORES_F32, _lib.FA_SCORES_REFERENCE)


def test_single_sequence_no_prefix(device):
    run_and_check(build(device, LLAMA8B, [300], [0], 1))


def test_chunk_boundaries(device):
    # lengths around multiples of the 64-token chunk and the 128-token KV tile
    run_and_check(build(device, LLAMA8B, [63, 64, 65, 127, 128, 129, 200], [0] * 7, 2))


def test_long_prefix_short_suffix(device):
    run_and_check(build(device, LLAMA8B, [1500, 900, 400], [1472, 640, 16], 3))


def test_empty_and_one_token_sequences(device):
    run_and_check(build(device, LLAMA8B, [40, 200, 77, 130, 90], [40, 199, 0, 64, 89], 4),
                  flows=BOTH)


@pytest.mark.parametrize("heads", [Heads(8, 8, 128), Heads(32, 4, 128), QWEN7B, Heads(16, 2, 128)])
def test_gqa_ratios(device, heads):
    run_and_check(build(device, heads, [260, 131, 75], [32, 0, 48], 5))


def test_f16_pool(device):
    run_and_check(build(device, LLAMA8B, [333, 150], [96, 0], 6, dtype=torch.float16), flows=BOTH)


@pytest.mark.parametrize("seed", [1003, 1004, 1005])
def test_c3_full_configuration(device, seed):
    run_and_check(make_c3(device, seed=seed), flows=BOTH)


def test_c5_prompt_shapes(device):
    # C5's new prompts: Qwen2-7B heads (n_rep 7), L ~ U[256, 2048], no cached prefix.
    lens = np.random.default_rng(55).integers(256, 2049, size=5)
    run_and_check(build(device, QWEN7B, lens, [0] * 5, 55), flows=BOTH)


def test_prefill_repeatable(device):
    b = build(device, LLAMA8B, [700, 500], [128, 0], 7)
    o1 = run_and_check(b).clone()
    o2 = run_and_check(b)
    assert torch.equal(o1, o2)


def test_many_sequences_share_one_persistent_launch(device):
    # 300 short sequences (more work items than SMs, several per CTA) plus a long one.
    rng = np.random.default_rng(9)
    lens = list(rng.integers(1, 90, size=300)) + [1700]
    prefix = [int(x) // 2 // 16 * 16 for x in lens]
    run_and_check(build(device, LLAMA8B, lens, prefix, 9))


def test_invalid_context_zeroes_rows_and_reports(device):
    b = build(device, LLAMA8B, [300, 200], [0, 0], 10)
    ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    ctx = b.context_lens.clone()
    ctx[0] = 100  # shorter than its 300 query tokens
    ops.device_status()
    out = ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, ctx,
                            b.block_tables, 4, 1 / math.sqrt(128), b.max_seqlen_q,
                            b.max_context_len, ops.Workspace(device))
    assert ops.device_status() & _lib.FA_DEVERR_CONTEXT
    assert float(out[:300].float().abs().sum()) == 0.0
    good = oracle_attention(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                            b.block_tables, 4, 1 / math.sqrt(128))
    assert max_abs(f32(out[300:]), good[300:]) <= TOL


def test_bad_block_id_reported(device):
    b = build(device, LLAMA8B, [300, 200], [0, 0], 8)
    ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    bt = b.block_tables.clone()
    bt[1, 2] = 1 << 20
    ops.device_status()
    ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens, bt, 4,
                      1 / math.sqrt(128), b.max_seqlen_q, b.max_context_len, ops.Workspace(device))
    assert ops.device_status() & _lib.FA_DEVERR_BLOCK_ID


@pytest.mark.parametrize("heads", [LLAMA8B, QWEN7B])
def test_prefix_reuse_leaves_suffix_rows_unchanged(device, heads):
    # The invariance the reference checks end to end (model.rs:244-360, 1e-4 in f32): a prompt
    # prefilled cold, and the same prompt prefilled as a suffix over its cached prefix, give the
    # suffix tokens the same attention output. Here on the tcgen05 path (bf16): both runs read
    # the same pool, so the outputs differ only by tile alignment (chunks start at different
    # tokens), far inside the bf16 tolerance.
    lens, P = [1000, 333], [512, 208]
    cold = build(device, heads, lens, [0, 0], seed=77)
    out_cold = run_and_check(cold)
    # Same pool, tables and Q/K/V; only the last len - P tokens are queries.
    h = heads
    scale = 1 / math.sqrt(h.head_dim)
    cu_cold = cold.cu_seqlens_q.cpu().numpy()
    rows = np.concatenate([np.arange(cu_cold[i] + P[i], cu_cold[i + 1]) for i in range(len(lens))])
    suffix = np.array(lens) - np.array(P)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(suffix)]), dtype=torch.int32, device=device)
    q = cold.q[torch.from_numpy(rows).to(device)].contiguous()
    out_warm = ops.paged_prefill(q, cold.k_caches[0], cold.v_caches[0], cu, cold.context_lens,
                                 cold.block_tables, h.n_rep, scale, int(suffix.max()),
                                 cold.max_context_len, ops.Workspace(device))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert max_abs(f32(out_warm), f32(out_cold)[rows]) <= 1e-2


def test_more_sequences_than_one_launch_holds(device):
    # A call with more than 2048 sequences runs as consecutive launches of the kernel on the
    # stream (its sequence table lives in shared memory), which share the workspace's work
    # counter and, with programmatic dependent launch, may be resident while the previous one
    # finishes: every launch must still see the counter at zero and cover its own sequences.
    rng = np.random.default_rng(71)
    n = 2300
    lens = rng.integers(1, 48, size=n)
    prefix = np.minimum(lens - 1, rng.integers(0, 20, size=n)) // 16 * 16
    b = build(device, Heads(8, 2, 128), lens, prefix, 72)
    out = run_and_check(b)
    # Once more on the same workspace: the counter came back to zero after the last launch.
    h = b.heads
    ws = ops.Workspace(device)
    for _ in range(2):
        again = ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q,
                                  b.context_lens, b.block_tables, h.n_rep,
                                  1 / math.sqrt(h.head_dim), b.max_seqlen_q, b.max_context_len, ws)
        torch.cuda.synchronize()
        assert torch.equal(again, out)
    assert ops.device_status() == 0
