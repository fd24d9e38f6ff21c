"""fa_paged_decode_append: the new token's K/V write and the decode attention in one launch.

The reference's decode step is Cache::write_kv of the new token followed by paged_attention
over the whole context (src/models/common/attention.rs:104-109). The fused entry point must leave
the pool and produce the output exactly as fa_reshape_and_cache (slots of position L-1) followed
by fa_paged_decode do: same kernel, same split plan, so both are compared bit for bit, and the
output is also checked against the oracle at the bf16 tolerance.
"""

import math

import numpy as np
import pytest
import torch

from flour_b200 import FlourAttnError, _lib, ops
from flour_b200.workloads import LLAMA8B, QWEN05, QWEN7B, c2_contexts, make_decode

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def new_token_slots(b):
    """Slot of position L-1 of every sequence (the reference's BlockTable::slot)."""
    bt = b.block_tables.cpu().numpy()
    last = b.ctx_host.astype(np.int64) - 1
    return torch.tensor(bt[np.arange(b.num_seqs), last // 16] * 16 + last % 16, dtype=torch.int32,
                        device=b.q.device)


def both_paths(heads, ctx, dtype, device, seed, key_view=None):
    """Run the fused call on one copy of a batch and the two-launch path on an identical copy."""
    fused = make_decode(heads, ctx, dtype, device, seed)
    split = make_decode(heads, ctx, dtype, device, seed)
    g = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (fused.num_seqs, heads.num_kv_heads, heads.head_dim)
    if key_view is None:
        key = torch.randn(shape, device=device, generator=g).to(dtype)
        value = torch.randn(shape, device=device, generator=g).to(dtype)
    else:
        key, value = key_view(shape, g)
    scale = 1.0 / math.sqrt(heads.head_dim)
    out = ops.paged_decode_append(fused.q, fused.k_caches[0], fused.v_caches[0], key, value,
                                  fused.block_tables, fused.context_lens, heads.n_rep, scale,
                                  fused.max_context_len, ops.Workspace(device))
    ops.reshape_and_cache(split.k_caches[0], split.v_caches[0], key, value, new_token_slots(split))
    want = ops.paged_decode(split.q, split.k_caches[0], split.v_caches[0], split.block_tables,
                            split.context_lens, heads.n_rep, scale, split.max_context_len,
                            ops.Workspace(device))
    torch.cuda.synchronize()
    return fused, split, out, want


def check_same(fused, split, out, want):
    assert ops.device_status() == 0
    assert torch.equal(fused.k_caches[0], split.k_caches[0]), "K pools differ"
    assert torch.equal(fused.v_caches[0], split.v_caches[0]), "V pools differ"
    assert torch.equal(out, want), "outputs differ from reshape_and_cache + paged_decode"
    h = fused.heads
    cu = torch.arange(fused.num_seqs + 1, dtype=torch.int32)
    ref = oracle_attention(fused.q, fused.k_caches[0], fused.v_caches[0], cu, fused.context_lens,
                           fused.block_tables, h.n_rep, 1.0 / math.sqrt(h.head_dim))
    assert max_abs(f32(out), ref) <= TOL_BF16


def test_c2_shapes_split_k(device):
    fused, split, out, want = both_paths(LLAMA8B, c2_contexts(31, batch=24), torch.bfloat16,
                                         device, 31)
    check_same(fused, split, out, want)


@pytest.mark.parametrize("heads,dtype", [(QWEN05, torch.float16), (QWEN7B, torch.bfloat16)])
def test_page_boundaries_and_short_contexts(device, heads, dtype):
    # L-1 on the first slot of a fresh page (17, 33, 4097), on the last slot (16, 4096), and L=1.
    ctx = np.array([1, 2, 16, 17, 33, 4096, 4097, 700])
    fused, split, out, want = both_paths(heads, ctx, dtype, device, 32)
    check_same(fused, split, out, want)


def test_strided_key_value(device):
    def views(shape, g):
        B, kvh, d = shape
        big = torch.randn((B, kvh, 3 * d), device=device, generator=g).to(torch.bfloat16)
        return big[:, :, d:2 * d], big[:, :, 2 * d:]  # token stride 3*kvh*d, head stride 3*d
    fused, split, out, want = both_paths(LLAMA8B, c2_contexts(33, batch=8), torch.bfloat16,
                                         device, 33, key_view=views)
    check_same(fused, split, out, want)


def test_invalid_context_writes_nothing(device):
    b = make_decode(LLAMA8B, np.array([300, 40]), torch.bfloat16, device, 34)
    k0, v0 = b.k_caches[0].clone(), b.v_caches[0].clone()
    key = torch.ones((2, 8, 128), dtype=torch.bfloat16, device=device)
    cl = b.context_lens.clone()
    cl[1] = 0
    ops.device_status()
    out = ops.paged_decode_append(b.q, b.k_caches[0], b.v_caches[0], key, key, b.block_tables, cl,
                                  4, 0.1, b.max_context_len, ops.Workspace(device))
    torch.cuda.synchronize()
    assert ops.device_status() & _lib.FA_DEVERR_CONTEXT
    assert not out[1].any()
    # Sequence 0 got its token at position 299; nothing else in the pool changed.
    changed = (b.k_caches[0] != k0).any(dim=(2, 3)).nonzero().tolist()
    blk = int(b.block_tables[0, 299 // 16])
    assert changed == [[blk, h] for h in range(8)]
    assert (b.v_caches[0] != v0).any(dim=(2, 3)).nonzero().tolist() == changed


def test_host_rejections(device):
    b = make_decode(LLAMA8B, np.array([64]), torch.float32, device, 35)
    key = torch.zeros((1, 8, 128), dtype=torch.float32, device=device)
    with pytest.raises(FlourAttnError) as e:
        ops.paged_decode_append(b.q, b.k_caches[0], b.v_caches[0], key, key, b.block_tables,
                                b.context_lens, 4, 0.1, 64, ops.Workspace(device))
    assert e.value.status == _lib.FA_EUNSUPPORTED
