"""The C-ABI library loads, exports every declared symbol, and rejects bad arguments on the
host before touching a GPU (no compute calls here)."""

import ctypes
import re

import pytest

from flour_b200 import _lib
from flour_b200._lib import FaKvLayer, lib


def declared_functions():
    text = _lib.HEADER_PATH.read_text()
    return sorted(set(re.findall(r"FA_API\s+[\w\s\*]*?\b(fa_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    decl = declared_functions()
    assert decl == sorted(_lib.SIGNATURES), (decl, sorted(_lib.SIGNATURES))
    assert len(decl) >= 12


def test_library_exports_every_declared_symbol():
    L = lib()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_library_is_built_for_sm100a():
    data = _lib.LIB_PATH.read_bytes()
    assert b"sm_100a" in data


def test_status_strings():
    L = lib()
    assert L.fa_abi_version() == 2
    assert L.fa_status_string(0) == b"ok"
    assert L.fa_status_string(-1) == b"invalid argument"
    assert L.fa_status_string(-6) == b"kernel reported bad device data"


def layer(nb=8, kvh=2, bs=16, d=64, dt=_lib.FA_BF16, k=0x1000, v=0x2000):
    return FaKvLayer(k, v, nb, kvh, bs, d, dt)


def test_host_validation_rejects_before_launch():
    L = lib()
    P = ctypes.c_void_p
    ly = layer()
    fake = P(0x10000)
    # NULL layer
    assert L.fa_paged_decode(None, fake, fake, fake, fake, 4, 1, 4, 2, 16, 0.1, 0, None, 0, None) == _lib.FA_EINVAL
    assert b"layer is NULL" in L.fa_last_error_message()
    # num_heads != n_rep * kv_heads (repeat_kv contract, cpu.rs:78-79)
    assert L.fa_paged_decode(ctypes.byref(ly), fake, fake, fake, fake, 4, 1, 5, 2, 16, 0.1, 0, None, 0, None) == _lib.FA_EINVAL
    assert b"n_rep" in L.fa_last_error_message()
    # context longer than the table can hold
    assert L.fa_paged_decode(ctypes.byref(ly), fake, fake, fake, fake, 4, 1, 4, 2, 65, 0.1, 0, None, 0, None) == _lib.FA_ERANGE
    # non-finite scale
    assert L.fa_paged_decode(ctypes.byref(ly), fake, fake, fake, fake, 4, 1, 4, 2, 16, float("nan"), 0, None, 0, None) == _lib.FA_EINVAL
    # unknown score flow
    assert L.fa_paged_decode(ctypes.byref(ly), fake, fake, fake, fake, 4, 1, 4, 2, 16, 0.1, 2, None, 0, None) == _lib.FA_EINVAL
    assert b"score_flow" in L.fa_last_error_message()
    # bad dtype
    bad = layer(dt=7)
    assert L.fa_reshape_and_cache(ctypes.byref(bad), fake, fake, 128, 64, 128, 64, fake, 3, None) == _lib.FA_EINVAL
    # write_block / read_block out of range (PagedKvPool rejects bad blocks)
    assert L.fa_write_block(ctypes.byref(ly), 8, fake, fake, None) == _lib.FA_ERANGE
    assert L.fa_read_block(ctypes.byref(ly), -1, fake, fake, None) == _lib.FA_ERANGE
    # copy_blocks layer-count bounds and shape agreement
    assert L.fa_copy_blocks(ctypes.byref(ly), 0, fake, 1, None) == _lib.FA_EINVAL
    two = (FaKvLayer * 2)(layer(), layer(d=128))
    assert L.fa_copy_blocks(two, 2, fake, 1, None) == _lib.FA_EINVAL
    # prefill: query longer than the context
    assert L.fa_paged_prefill(ctypes.byref(ly), fake, fake, fake, fake, fake, 4, 1, 4, 2, 8, 8, 4, 0.1, 0, None, 0, None) == _lib.FA_ERANGE
    # empty work is a no-op success
    assert L.fa_reshape_and_cache(ctypes.byref(ly), fake, fake, 128, 64, 128, 64, fake, 0, None) == _lib.FA_OK
    assert L.fa_copy_blocks(ctypes.byref(ly), 1, fake, 0, None) == _lib.FA_OK


def test_workspace_sizes():
    L = lib()
    # Prefill needs only its two work counters.
    assert L.fa_paged_attention_workspace_size(16, 32, 8, 128, 2048, 2048) == 256
    # C2 decode: 64 sequences x 8 kv heads, contexts up to 4096 -> split-K partials.
    ws = L.fa_paged_attention_workspace_size(64, 32, 8, 128, 4096, 1)
    assert ws > 64 * 32 * 128 * 4
    # C4 long context needs more splits -> a larger workspace.
    assert L.fa_paged_attention_workspace_size(16, 32, 8, 128, 32768, 1) > 16 * 32 * 128 * 4 * 4
    assert L.fa_paged_attention_workspace_size(0, 32, 8, 128, 4096, 1) == 0


def _decode_plan_workspace(num_seqs, num_heads, num_kv_heads, head_dim, max_context_len):
    """The decode split plan and its workspace, restated: about 12 CTAs per SM over 148 SMs for
    the longest context, 32 to 256 pages per split rounded up to a multiple of 4; then merge
    tickets, per-split LSE and per-split f32 partial outputs, each region 256-byte aligned."""
    r256 = lambda x: (x + 255) // 256 * 256
    max_pages = -(-max_context_len // 16)
    units = num_seqs * num_kv_heads
    want = max(1, -(-148 * 12 // units))
    pps = min((max(-(-max_pages // want), 32) + 3) // 4 * 4, 256)
    splits = max(-(-max_pages // pps), 1)
    if splits <= 1:
        return pps, splits, 0
    lse_off = r256(num_seqs * num_kv_heads * 4)
    o_off = lse_off + r256(num_seqs * num_heads * splits * 4)
    return pps, splits, o_off + num_seqs * num_heads * splits * head_dim * 4


@pytest.mark.parametrize("shape, pps, splits", [
    ((64, 32, 8, 128, 4096), 64, 4),      # C2 batch
    ((59, 28, 4, 128, 6438), 52, 8),      # a C5 rank's decode share at N=8
    ((59, 28, 4, 128, 1419), 32, 3),      # short uniform contexts: the 32-page floor
    ((16, 32, 8, 128, 32768), 148, 14),   # C4 long context
    ((4, 32, 8, 128, 256), 32, 1),        # one split: no workspace
])
def test_decode_split_plan_is_pinned(shape, pps, splits):
    """The measured-best split plan (C2, C5 shares, short batches, C4) is what the library
    sizes its workspace for; a retuned plan must change these cases on purpose."""
    got_pps, got_splits, expect = _decode_plan_workspace(*shape)
    assert (got_pps, got_splits) == (pps, splits)
    assert lib().fa_paged_attention_workspace_size(*shape, 1) == expect


def test_decode_workspace_too_small_is_rejected_without_launch():
    L = lib()
    ly = layer(nb=4096, kvh=8, bs=16, d=128)
    fake = ctypes.c_void_p(0x10000)
    need = L.fa_paged_attention_workspace_size(64, 32, 8, 128, 4096, 1)
    assert need > 0
    st = L.fa_paged_decode(ctypes.byref(ly), fake, fake, fake, fake, 256, 64, 32, 4, 4096, 0.1,
                           0, ctypes.c_void_p(0x100000), need - 1, None)
    assert st == _lib.FA_ERANGE
    assert b"workspace" in L.fa_last_error_message()


def test_workspace_reset_rejects_null_and_accepts_any_pointer():
    L = lib()
    assert L.fa_workspace_reset(None) == _lib.FA_EINVAL
    assert b"NULL" in L.fa_last_error_message()
    # Forgetting a pointer the library never saw is a no-op success (host bookkeeping only).
    assert L.fa_workspace_reset(ctypes.c_void_p(0x123400)) == _lib.FA_OK
