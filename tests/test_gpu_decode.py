"""Paged decode on the GPU against the oracle (src/backend/cpu.rs:57-112 with seq_q = 1).

Tolerances (from the north star): max-abs 1e-5 for f32 pools (f32 accumulate everywhere),
2e-2 for bf16/f16 pools (bf16 output rounding plus the bf16 rounding of the probabilities
fed to the tensor cores)."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import FlourAttnError, _lib, ops
from flour_b200.paged import KvCache, paged_attention
from flour_b200.workloads import (LLAMA8B, QWEN05, QWEN7B, Heads, c2_contexts, make_c1,
                                  make_decode)

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_BF16 = 2e-2


def run_decode(batch, ws=None, max_context_len=None, score_flow=_lib.FA_SCORES_F32):
    h = batch.heads
    ws = ws or ops.Workspace(batch.q.device)
    return ops.paged_decode(batch.q, batch.k_caches[0], batch.v_caches[0], batch.block_tables,
                            batch.context_lens, h.n_rep, 1.0 / math.sqrt(h.head_dim),
                            max_context_len or batch.max_context_len, ws, score_flow=score_flow)


def check_both_flows(batch, tol):
    """The default flow against f32-score oracle (score_mode 0), and FA_SCORES_REFERENCE
    against the reference's dtype flow (score_mode 1, cpu.rs:84-85)."""
    check(batch, run_decode(batch), tol, score_modes=(0,))
    check(batch, run_decode(batch, score_flow=_lib.FA_SCORES_REFERENCE), tol, score_modes=(1,))


def check(batch, out, tol, score_modes=(0,)):
    h = batch.heads
    B = batch.num_seqs
    cu = torch.arange(B + 1, dtype=torch.int32)
    for mode in score_modes:
        want = oracle_attention(batch.q, batch.k_caches[0], batch.v_caches[0], cu,
                                batch.context_lens, batch.block_tables, h.n_rep,
                                1.0 / math.sqrt(h.head_dim), score_mode=mode)
        err = max_abs(f32(out), want)
        assert err <= tol, f"score_mode {mode}: max-abs {err} > {tol}"
    assert ops.device_status() == 0


def test_c1_qwen05_f32(device):
    b = make_c1(device, seed=1)
    check(b, run_decode(b), TOL_F32)


@pytest.mark.parametrize("seed", [2, 3])
def test_c2_llama8b_bf16(device, seed):
    b = make_decode(LLAMA8B, c2_contexts(seed, batch=8), torch.bfloat16, device, seed)
    check_both_flows(b, TOL_BF16)


def test_c2_full_batch_against_oracle(device):
    # All 64 sequences of the benchmark configuration (one layer).
    b = make_decode(LLAMA8B, c2_contexts(1234), torch.bfloat16, device, 1234)
    check_both_flows(b, TOL_BF16)


def test_c4_long_context_split_k(device):
    ctx = np.random.default_rng(4).integers(16384, 32769, size=2)
    b = make_decode(LLAMA8B, ctx, torch.bfloat16, device, 4)
    check_both_flows(b, TOL_BF16)


def test_c5_qwen7b_heads_n_rep_7(device):
    ctx = np.random.default_rng(5).integers(1, 3000, size=12)
    b = make_decode(QWEN7B, ctx, torch.bfloat16, device, 5)
    check_both_flows(b, TOL_BF16)


def test_c5_decode_context_distribution(device):
    # C5's decode contexts: LogNormal(ln 1024, 0.8) capped at 8192, Qwen2-7B heads.
    from flour_b200.workloads import c5_contexts
    b = make_decode(QWEN7B, c5_contexts(56, 24), torch.bfloat16, device, 56)
    check_both_flows(b, TOL_BF16)


@pytest.mark.parametrize("heads", [QWEN05, Heads(8, 8, 128), Heads(16, 2, 128)])
def test_other_head_shapes_bf16(device, heads):
    ctx = np.random.default_rng(6).integers(1, 1200, size=5)
    b = make_decode(heads, ctx, torch.bfloat16, device, 6)
    check(b, run_decode(b), TOL_BF16)


def test_f16_pool(device):
    ctx = np.random.default_rng(7).integers(1, 2500, size=6)
    b = make_decode(LLAMA8B, ctx, torch.float16, device, 7)
    check_both_flows(b, TOL_BF16)


def test_f32_llama_shapes_generic_path(device):
    ctx = np.random.default_rng(8).integers(1, 700, size=3)
    b = make_decode(LLAMA8B, ctx, torch.float32, device, 8, value_scale=0.125)
    check(b, run_decode(b), TOL_F32)
    # For f32 pools the reference flow rounds nothing: the same bits as the default flow.
    assert torch.equal(run_decode(b, score_flow=_lib.FA_SCORES_REFERENCE), run_decode(b))


def test_bf16_generic_path_reference_flow(device):
    # block_size 8 takes the generic kernel; its reference flow against score_mode 1.
    h = Heads(8, 2, 96, block_size=8)
    ctx = np.random.default_rng(18).integers(1, 900, size=4)
    b = make_decode(h, ctx, torch.bfloat16, device, 18)
    check_both_flows(b, TOL_BF16)


@pytest.mark.parametrize("ctx", [[1], [15], [16], [17], [1, 16, 17, 33], [255, 256, 257]])
def test_edge_context_lengths(device, ctx):
    b = make_decode(LLAMA8B, np.array(ctx), torch.bfloat16, device, 9, pool_blocks=64)
    check(b, run_decode(b), TOL_BF16)


def test_split_count_does_not_change_result_and_repeats_are_identical(device):
    ctx = np.random.default_rng(10).integers(2000, 9000, size=4)
    b = make_decode(LLAMA8B, ctx, torch.bfloat16, device, 10)
    ws = ops.Workspace(device)
    o1 = run_decode(b, ws).clone()
    o2 = run_decode(b, ws).clone()  # merge tickets were reset by the first call
    assert torch.equal(o1, o2)
    # A larger host bound changes the split plan; the result stays within tolerance.
    o3 = run_decode(b, ops.Workspace(device), max_context_len=b.block_tables.shape[1] * 16)
    assert max_abs(f32(o1), f32(o3)) <= TOL_BF16
    check(b, o3, TOL_BF16)


def test_workspace_reused_across_shapes(device):
    # A few long sequences leave split-K partials right after their small ticket region; a
    # larger batch then puts its tickets there. Results must equal runs on fresh workspaces,
    # eagerly and when the small call is replayed from a CUDA graph in between.
    small = make_decode(LLAMA8B, np.array([9000, 7000, 8000, 6000]), torch.bfloat16, device, 14)
    big = make_decode(LLAMA8B, c2_contexts(15, batch=64), torch.bfloat16, device, 15)
    want_small = run_decode(small, ops.Workspace(device)).clone()
    want_big = run_decode(big, ops.Workspace(device)).clone()
    ws = ops.Workspace(device)
    ws.get(64 << 20)  # one buffer for every call below
    for _ in range(2):
        assert torch.equal(run_decode(small, ws), want_small)
        assert torch.equal(run_decode(big, ws), want_big)
    out = torch.empty_like(small.q)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.paged_decode(small.q, small.k_caches[0], small.v_caches[0], small.block_tables,
                         small.context_lens, 4, 1.0 / math.sqrt(128), small.max_context_len, ws,
                         out=out)
    for _ in range(2):
        graph.replay()
        assert torch.equal(out, want_small)
        assert torch.equal(run_decode(big, ws), want_big)
    del graph
    assert ops.device_status() == 0


def _memsets_during(fn):
    """Number of device memsets that `fn` enqueues (CUDA activity trace)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    # Device-side activity only (the runtime API call is listed as a separate cudaMemsetAsync).
    return sum(1 for e in prof.events()
               if "memset" in e.name.lower() and not e.name.startswith("cuda"))


def test_workspace_ticket_zeroing_is_paid_once(device):
    # Eager large, small, large, large on one workspace: the first large call after the small one
    # zeroes the tickets that land on the small call's partials; the next large call finds them
    # clean and issues no memset. Every output equals a run on a fresh workspace.
    small = make_decode(LLAMA8B, np.array([9000, 7000, 8000, 6000]), torch.bfloat16, device, 16)
    big = make_decode(LLAMA8B, c2_contexts(17, batch=64), torch.bfloat16, device, 17)
    want_small = run_decode(small, ops.Workspace(device)).clone()
    want_big = run_decode(big, ops.Workspace(device)).clone()
    ws = ops.Workspace(device)
    ws.get(64 << 20)
    assert torch.equal(run_decode(big, ws), want_big)
    assert torch.equal(run_decode(small, ws), want_small)
    got = {}
    n1 = _memsets_during(lambda: got.setdefault("a", run_decode(big, ws).clone()))
    n2 = _memsets_during(lambda: got.setdefault("b", run_decode(big, ws).clone()))
    assert torch.equal(got["a"], want_big) and torch.equal(got["b"], want_big)
    assert (n1, n2) == (1, 0)
    assert ops.device_status() == 0


def test_general_entry_dispatches_decode(device):
    ctx = np.random.default_rng(12).integers(100, 3000, size=6)
    b = make_decode(LLAMA8B, ctx, torch.bfloat16, device, 12)
    B = b.num_seqs
    cu = torch.arange(B + 1, dtype=torch.int32, device=device)
    out = ops.paged_attention_varlen(b.q, b.k_caches[0], b.v_caches[0], cu, b.context_lens,
                                     b.block_tables, 4, 1 / math.sqrt(128), 1, b.max_context_len,
                                     ops.Workspace(device))
    assert torch.equal(out, run_decode(b))


def test_bad_block_id_and_context_are_reported(device):
    b = make_decode(LLAMA8B, np.array([40, 50]), torch.bfloat16, device, 13, pool_blocks=16)
    ops.device_status()
    bt = b.block_tables.clone()
    bt[0, 1] = 10_000
    ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], bt, b.context_lens, 4, 0.1, 64,
                     ops.Workspace(device))
    assert ops.device_status() & _lib.FA_DEVERR_BLOCK_ID
    ctx = b.context_lens.clone()
    ctx[1] = 10_000  # beyond max_blocks_per_seq * 16
    out = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, ctx, 4, 0.1, 64,
                           ops.Workspace(device))
    assert ops.device_status() & _lib.FA_DEVERR_CONTEXT
    assert float(out[1].float().abs().sum()) == 0.0


def test_host_rejections(device):
    b = make_decode(LLAMA8B, np.array([40]), torch.bfloat16, device, 14)
    with pytest.raises(FlourAttnError) as e:
        ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens, 3,
                         0.1, 40, ops.Workspace(device))
    assert e.value.status == _lib.FA_EINVAL


def test_kv_cache_mirror_decode_steps(device):
    # Engine-style use of the mirror: prefill 37 tokens, then 3 decode steps, each doing
    # allocate_kv -> write_kv -> kv_blocks -> paged_attention (attention.rs:104-109).
    torch.manual_seed(0)
    hq, hkv, d = 32, 8, 128
    cache = KvCache(1, 256, hkv, d, torch.bfloat16, device)
    cache.allocate_kv(37)
    k = torch.randn((1, hkv, 37, d), device=device).to(torch.bfloat16)
    cache.write_kv(0, k, k * 0.5)
    dense_k, dense_v = [k], [k * 0.5]
    for step in range(3):
        cache.allocate_kv(1)
        kn = torch.randn((1, hkv, 1, d), device=device).to(torch.bfloat16)
        cache.write_kv(0, kn, kn + 1)
        dense_k.append(kn)
        dense_v.append(kn + 1)
        q = torch.randn((1, hq, 1, d), device=device).to(torch.bfloat16)
        out = paged_attention(q, cache.kv_blocks(0), hq // hkv, 1 / math.sqrt(d))
        kk = torch.cat(dense_k, 2)[0].float()
        vv = torch.cat(dense_v, 2)[0].float()
        ref = torch.softmax((q[0].float() @ kk.repeat_interleave(4, 0).transpose(1, 2)) / math.sqrt(d), -1) \
            @ vv.repeat_interleave(4, 0)
        assert out.shape == q.shape
        assert max_abs(f32(out[0]), ref.cpu().numpy()) <= TOL_BF16
