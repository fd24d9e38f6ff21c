"""The C5 mixed serving step as the benchmark runs it: decode sequences (new token written and
attended in one fa_paged_decode_append launch per layer) on one stream and new prompts
(fa_reshape_and_cache + fa_paged_prefill per layer) on a second stream, forked and joined inside
the step, eagerly and replayed from a CUDA graph. Both sub-batches' outputs are compared with the
oracle restatement of src/backend/cpu.rs:57-112 in both score flows (f32 scores, and the
reference's bf16 dtype flow of cpu.rs:84-85, each kernel flow against its oracle mode), at a
reduced size: Qwen2-7B heads, C5's context
and prompt-length distributions, 2 layers."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import _lib, ops
from flour_b200.workloads import QWEN7B, c5_contexts, make_mixed_step

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu
TOL = 2e-2
LAYERS = 2


def check_step(ms):
    """Outputs against the oracle in the score flow the step ran with (FA_SCORES_F32 <->
    score_mode 0, FA_SCORES_REFERENCE <-> score_mode 1)."""
    h = ms.heads
    scale = 1 / math.sqrt(h.head_dim)
    last = ms.num_layers - 1  # every layer writes the same outputs; the last one remains
    d, p = ms.dec, ms.pf
    for mode in (ms.score_flow,):
        cu = torch.arange(d.num_seqs + 1, dtype=torch.int32)
        want = oracle_attention(d.q, d.k_caches[last], d.v_caches[last], cu, d.context_lens,
                                d.block_tables, h.n_rep, scale, score_mode=mode)
        err = max_abs(f32(ms.dout), want)
        assert err <= TOL, f"decode, score_mode {mode}: max-abs {err}"
        want = oracle_attention(p.q, p.k_caches[last], p.v_caches[last], p.cu_seqlens_q,
                                p.context_lens, p.block_tables, h.n_rep, scale, score_mode=mode)
        err = max_abs(f32(ms.pout), want)
        assert err <= TOL, f"prefill, score_mode {mode}: max-abs {err}"
    # The fused append wrote each decode sequence's new K/V into its last slot in every layer.
    bt = d.block_tables.cpu().numpy()
    pos = d.ctx_host - 1
    blk, off = bt[np.arange(d.num_seqs), pos // 16], pos % 16
    for l in range(ms.num_layers):
        assert torch.equal(d.k_caches[l][blk, :, off], ms.dk)
        assert torch.equal(d.v_caches[l][blk, :, off], ms.dv)
    assert ops.device_status() == 0


@pytest.mark.parametrize("seed,flow", [(60, _lib.FA_SCORES_F32), (61, _lib.FA_SCORES_F32),
                                       (61, _lib.FA_SCORES_REFERENCE)])
def test_mixed_step_two_streams_eager_and_graph(device, seed, flow):
    rng = np.random.default_rng(seed)
    dec_ctx = c5_contexts(seed, 40)
    pf_len = rng.integers(256, 2049, size=4)
    ms = make_mixed_step(QWEN7B, dec_ctx, pf_len, torch.bfloat16, device, seed, LAYERS)
    ms.score_flow = flow
    ms.run()
    torch.cuda.synchronize()
    check_step(ms)
    eager = (ms.dout.clone(), ms.pout.clone())
    ms.dout.fill_(float("nan"))
    ms.pout.fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ms.run()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    del graph
    assert torch.equal(ms.dout, eager[0]) and torch.equal(ms.pout, eager[1])
    check_step(ms)
