"""A decode step of two layers run back to back without host synchronisation: fused QKV + RoPE +
cache write (fa_qkv_rope_cache), paged decode (fa_paged_decode), fused o_proj + residual
(fa_o_proj_residual), the next layer reading the residual stream, and the last-token logits
(fa_last_token_logits) of the final residual. The GEMMs and the decode are
launched with programmatic dependent launch, so each may start while its predecessor finishes;
their waits must keep every dependency (q and the written cache slots into the decode, the
attention output into o_proj, the residual stream into the next layer's QKV). The results must be
bit-identical to the same calls with a device synchronisation after each one, eagerly and
replayed from a CUDA graph."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import ops
from flour_b200.paged import rope_tables
from flour_b200.workloads import Heads, make_decode

pytestmark = pytest.mark.gpu

LAYERS = 2


def build(device):
    heads = Heads(8, 2, 128)
    hidden, B = 1024, 16
    ctx = np.random.default_rng(90).integers(100, 900, size=B)
    b = make_decode(heads, ctx, torch.bfloat16, device, 90, num_layers=LAYERS)
    g = torch.Generator(device=device).manual_seed(91)
    n_qkv = (heads.num_heads + 2 * heads.num_kv_heads) * heads.head_dim
    wqkv = [(torch.randn(n_qkv, hidden, device=device, generator=g) / 32).to(torch.bfloat16)
            for _ in range(LAYERS)]
    wo = [(torch.randn(hidden, heads.num_heads * heads.head_dim, device=device, generator=g) / 32)
          .to(torch.bfloat16) for _ in range(LAYERS)]
    x0 = torch.randn(B, hidden, device=device, generator=g).to(torch.bfloat16)
    pos = torch.tensor(ctx - 1, dtype=torch.int32, device=device)
    bt = b.block_tables.cpu().numpy()
    slots = torch.tensor(bt[np.arange(B), (ctx - 1) // 16] * 16 + (ctx - 1) % 16,
                         dtype=torch.int32, device=device)
    cos, sin = rope_tables(heads.head_dim, 4096, 500000.0, torch.bfloat16, device)
    bufs = {"q": torch.empty(B, heads.num_heads, heads.head_dim, device=device,
                             dtype=torch.bfloat16),
            "attn": torch.empty(B, heads.num_heads, heads.head_dim, device=device,
                                dtype=torch.bfloat16),
            "x": [torch.empty_like(x0) for _ in range(LAYERS)]}
    lm_head = (torch.randn(4096, hidden, device=device, generator=g) / 32).to(torch.bfloat16)
    norm_w = (1 + torch.randn(hidden, device=device, generator=g) / 8).to(torch.bfloat16)
    bufs["cu"] = torch.arange(B + 1, dtype=torch.int32, device=device)
    bufs["logits"] = torch.empty(B, 4096, device=device, dtype=torch.float32)
    ws = ops.Workspace(device)
    ws.get(ops.workspace_size(B, heads.num_heads, heads.num_kv_heads, heads.head_dim,
                              b.max_context_len, 1))
    return heads, b, wqkv, wo, x0, pos, slots, cos, sin, bufs, ws, lm_head, norm_w


def step(env, sync):
    heads, b, wqkv, wo, x0, pos, slots, cos, sin, bufs, ws, lm_head, norm_w = env
    x = x0
    for l in range(LAYERS):
        ops.qkv_rope_cache(x, wqkv[l], b.k_caches[l], b.v_caches[l], pos, slots,
                           heads.num_heads, cos, sin, q_out=bufs["q"])
        if sync:
            torch.cuda.synchronize()
        ops.paged_decode(bufs["q"], b.k_caches[l], b.v_caches[l], b.block_tables, b.context_lens,
                         heads.n_rep, 1 / math.sqrt(heads.head_dim), b.max_context_len, ws,
                         out=bufs["attn"])
        if sync:
            torch.cuda.synchronize()
        ops.o_proj_residual(bufs["attn"].reshape(x.shape[0], -1), wo[l], x, out=bufs["x"][l])
        if sync:
            torch.cuda.synchronize()
        x = bufs["x"][l]
    ops.last_token_logits(x, bufs["cu"], lm_head, norm_w, logits_out=bufs["logits"])
    return x


def test_layers_back_to_back_equal_synchronised_calls(device):
    env = build(device)
    want = step(env, sync=True).clone()
    bufs = env[9]
    want_q, want_attn, want_logits = bufs["q"].clone(), bufs["attn"].clone(), bufs["logits"].clone()
    for _ in range(2):
        got = step(env, sync=False)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert torch.equal(bufs["q"], want_q) and torch.equal(bufs["attn"], want_attn)
        assert torch.equal(bufs["logits"], want_logits)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(env, sync=False)
    for _ in range(3):
        for t in (bufs["q"], bufs["attn"], bufs["x"][0], bufs["x"][1], bufs["logits"]):
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(bufs["x"][-1], want) and torch.equal(bufs["logits"], want_logits)
    del graph
    assert ops.device_status() == 0
