"""fa_paged_decode_noalloc: decode for callers that cannot allocate device memory.

Such callers (an engine whose KV pool already fills the GPU and forbids allocation while
serving, or a host runtime that reaches the GPU only through this C ABI and owns no device
allocator) cannot provide the split-K workspace fa_paged_decode takes. The no-allocation entry
point uses the library's fixed device buffer instead. It must give the same results as the
workspace entry point (same kernel, same split plan), on two calls in a row (the buffer keeps
the previous call's contents, so its merge tickets are cleared by every call).

This file is named so pytest collects it last; it also passes alone in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from flour_b200 import FlourAttnError, _lib, ops
from flour_b200._lib import lib
from flour_b200.workloads import LLAMA8B, QWEN7B, c2_contexts, make_decode

from _util import f32, max_abs

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2  # the tolerance every bf16 decode parity test uses


def call_noalloc(b, out):
    """The new entry point through the C ABI, with the caller's stream."""
    layer = ops.layer_desc(b.k_caches[0], b.v_caches[0])
    st = lib().fa_paged_decode_noalloc(
        ctypes.byref(layer), ctypes.c_void_p(b.q.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(b.context_lens.data_ptr()), ctypes.c_void_p(b.block_tables.data_ptr()),
        b.block_tables.shape[1], b.num_seqs, b.heads.num_heads, b.heads.n_rep,
        b.max_context_len, 1.0 / math.sqrt(b.heads.head_dim),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "fa_paged_decode_noalloc")


def test_noalloc_decode_matches_workspace_decode_twice(device):
    # 24 sequences with contexts up to 4096: the split plan uses several splits, so the fixed
    # scratch buffer carries the partials and the merge tickets.
    b = make_decode(LLAMA8B, c2_contexts(77, batch=24), torch.bfloat16, device, 77)
    assert ops.workspace_size(b.num_seqs, 32, 8, 128, b.max_context_len, 1) > 0
    want = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens,
                            4, 1 / math.sqrt(128), b.max_context_len, ops.Workspace(device))
    for _ in range(2):
        out = torch.full_like(b.q, float("nan"))
        call_noalloc(b, out)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert max_abs(f32(out), f32(want)) <= TOL_BF16
        assert torch.equal(out, want)  # same kernel and split plan: identical bits


def test_noalloc_decode_rejects_requests_beyond_its_buffer(device):
    # 512 sequences of 32768 tokens need far more split-K scratch than the fixed buffer holds.
    b = make_decode(LLAMA8B, np.array([40]), torch.bfloat16, device, 78)
    layer = ops.layer_desc(b.k_caches[0], b.v_caches[0])
    fake = ctypes.c_void_p(b.q.data_ptr())
    need = ops.workspace_size(512, 32, 8, 128, 32768, 1)
    assert need > _lib.FA_NOALLOC_DECODE_SCRATCH_BYTES
    st = lib().fa_paged_decode_noalloc(ctypes.byref(layer), fake, fake, fake, fake, 2048, 512, 32,
                                       4, 32768, 0.1, None)
    assert st == _lib.FA_ERANGE
    assert b"scratch" in lib().fa_last_error_message()
    with pytest.raises(FlourAttnError):
        _lib.check(st, "fa_paged_decode_noalloc")


def test_noalloc_decode_after_calls_of_other_shapes(device):
    # The buffer keeps each call's partials right after its merge tickets. A call with more
    # (sequence, KV head) units puts its tickets where an earlier smaller call left partials,
    # and the other way round; every call must still equal the workspace entry point.
    small = make_decode(LLAMA8B, c2_contexts(79, batch=8), torch.bfloat16, device, 79)
    big = make_decode(LLAMA8B, c2_contexts(80, batch=64), torch.bfloat16, device, 80)
    qwen = make_decode(QWEN7B, c2_contexts(81, batch=8), torch.bfloat16, device, 81)
    want = {}
    for name, b in (("small", small), ("big", big), ("qwen", qwen)):
        h = b.heads
        assert ops.workspace_size(b.num_seqs, h.num_heads, h.num_kv_heads, h.head_dim,
                                  b.max_context_len, 1) > 0
        want[name] = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                      b.context_lens, h.n_rep, 1 / math.sqrt(h.head_dim),
                                      b.max_context_len, ops.Workspace(device))
    for name, b in (("small", small), ("big", big), ("qwen", qwen), ("big", big),
                    ("small", small)):
        out = torch.full_like(b.q, float("nan"))
        call_noalloc(b, out)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert torch.equal(out, want[name]), name


def test_noalloc_limit_is_the_workspace_size(device):
    # A call is accepted exactly when fa_paged_attention_workspace_size(..., max_seqlen_q=1)
    # fits the built-in buffer. Find batch sizes on either side of the limit (contexts planned
    # for up to 8192 tokens) and check both outcomes.
    limit = _lib.FA_NOALLOC_DECODE_SCRATCH_BYTES
    max_ctx = 8192
    sizes = {n: ops.workspace_size(n, 32, 8, 128, max_ctx, 1) for n in range(1, 600)}
    fits = max(n for n, sz in sizes.items() if sz <= limit)
    over = min(n for n, sz in sizes.items() if sz > limit)
    rng = np.random.default_rng(82)
    for n, accepted in ((fits, True), (over, False)):
        ctx = rng.integers(1, 48, size=n)
        ctx[0] = max_ctx  # the plan is made for the largest context
        b = make_decode(LLAMA8B, ctx, torch.bfloat16, device, 82)
        assert b.max_context_len == max_ctx
        out = torch.zeros_like(b.q)
        if accepted:
            call_noalloc(b, out)
            torch.cuda.synchronize()
            want = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                    b.context_lens, 4, 1 / math.sqrt(128), max_ctx,
                                    ops.Workspace(device))
            assert torch.equal(out, want)
        else:
            with pytest.raises(FlourAttnError) as ei:
                call_noalloc(b, out)
            assert ei.value.status == _lib.FA_ERANGE
    assert ops.device_status() == 0
