"""Maximum sizes: a pool whose K/V slabs hold more than 2^31 elements (element offsets of the
used blocks do not fit in 32 bits), and a prefill over a long cached prefix. Parity against the
oracle (src/backend/cpu.rs:57-112) on a compact copy of the blocks the tables use; block writes
and copies at those offsets are bit-exact."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import ops

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu
TOL = 2e-2
NB = 140_000  # 140000 x 8 x 16 x 128 = 2.29e9 elements per slab (> 2^31), 4.6 GB each (bf16)


@pytest.fixture(scope="module")
def big_pool(device):
    free, _ = torch.cuda.mem_get_info(device)
    need = 2 * NB * 8 * 16 * 128 * 2
    if free < need + (4 << 30):
        pytest.skip(f"needs {need / 1e9:.1f} GB free on the device")
    kc = torch.empty((NB, 8, 16, 128), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    yield kc, vc
    del kc, vc
    torch.cuda.empty_cache()


def compact(kc, vc, bt, ctx):
    """The blocks the tables use, copied into a small pool, and the tables remapped to it."""
    pages = (ctx + 15) // 16
    used = np.unique(np.concatenate([bt[i, :n] for i, n in enumerate(pages)]))
    remap = {int(b): i for i, b in enumerate(used)}
    bt2 = np.zeros_like(bt)
    for i, n in enumerate(pages):
        bt2[i, :n] = [remap[int(b)] for b in bt[i, :n]]
    idx = torch.from_numpy(used.astype(np.int64)).to(kc.device)
    return kc[idx].contiguous(), vc[idx].contiguous(), torch.from_numpy(bt2).to(kc.device)


def fill(cache, ids, gen):
    idx = torch.from_numpy(np.asarray(ids, np.int64)).to(cache.device)
    cache[idx] = torch.randn((len(ids),) + tuple(cache.shape[1:]), device=cache.device,
                             generator=gen).to(cache.dtype)


def test_decode_on_blocks_past_2g_elements(device, big_pool):
    kc, vc = big_pool
    rng = np.random.default_rng(21)
    ctx = np.array([3000, 1500, 33, 4096])
    pages = (ctx + 15) // 16
    ids = rng.choice(np.arange(NB - 3000, NB), size=int(pages.sum()), replace=False).astype(np.int32)
    bt = np.zeros((len(ctx), int(pages.max())), np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = ids[o:o + n]
        o += n
    g = torch.Generator(device=device).manual_seed(21)
    fill(kc, ids, g)
    fill(vc, ids, g)
    q = torch.randn((len(ctx), 32, 128), device=device, generator=g).to(torch.bfloat16)
    bt_d = torch.from_numpy(bt).to(device)
    ctx_d = torch.from_numpy(ctx.astype(np.int32)).to(device)
    scale = 1 / math.sqrt(128)
    out = ops.paged_decode(q, kc, vc, bt_d, ctx_d, 4, scale, int(ctx.max()), ops.Workspace(device))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    kc2, vc2, bt2 = compact(kc, vc, bt, ctx)
    cu = torch.arange(len(ctx) + 1, dtype=torch.int32, device=device)
    want = oracle_attention(q, kc2, vc2, cu, ctx_d, bt2, 4, scale)
    assert max_abs(f32(out), want) <= TOL


def test_block_writes_and_prefill_past_2g_elements(device, big_pool):
    kc, vc = big_pool
    rng = np.random.default_rng(22)
    lens, prefix = np.array([1500, 700]), np.array([1024, 0])
    pages = (lens + 15) // 16
    ids = rng.choice(np.arange(NB - 400, NB), size=int(pages.sum()), replace=False).astype(np.int32)
    bt = np.zeros((2, int(pages.max())), np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = ids[o:o + n]
        o += n
    g = torch.Generator(device=device).manual_seed(22)
    # cached prefix blocks get random values; the suffix comes through reshape_and_cache
    pre = [int(b) for i in range(2) for b in bt[i, :prefix[i] // 16]]
    if pre:
        fill(kc, pre, g)
        fill(vc, pre, g)
    suffix = lens - prefix
    T = int(suffix.sum())
    slots = np.concatenate([bt[i, np.arange(prefix[i], lens[i]) // 16] * 16 +
                            np.arange(prefix[i], lens[i]) % 16 for i in range(2)]).astype(np.int32)
    key = torch.randn((T, 8, 128), device=device, generator=g).to(torch.bfloat16)
    val = torch.randn((T, 8, 128), device=device, generator=g).to(torch.bfloat16)
    ops.reshape_and_cache(kc, vc, key, val, torch.from_numpy(slots).to(device))
    torch.cuda.synchronize()
    # bit-exact placement at 64-bit offsets
    s = torch.from_numpy(slots.astype(np.int64)).to(device)
    assert torch.equal(kc[s // 16, :, s % 16, :], key)
    assert torch.equal(vc[s // 16, :, s % 16, :], val)
    q = torch.randn((T, 32, 128), device=device, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0, int(suffix[0]), T], dtype=torch.int32, device=device)
    ctx_d = torch.from_numpy(lens.astype(np.int32)).to(device)
    scale = 1 / math.sqrt(128)
    out = ops.paged_prefill(q, kc, vc, cu, ctx_d, torch.from_numpy(bt).to(device), 4, scale,
                            int(suffix.max()), int(lens.max()), ops.Workspace(device))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    kc2, vc2, bt2 = compact(kc, vc, bt, lens)
    want = oracle_attention(q, kc2, vc2, cu, ctx_d, bt2, 4, scale)
    assert max_abs(f32(out), want) <= TOL
    # copy_blocks between two high blocks, bit-exact, other blocks untouched
    src, dst = int(ids[0]), NB - 1 if int(ids[0]) != NB - 1 else NB - 2
    before = kc[dst - 1].clone() if dst - 1 not in ids else None
    ops.copy_blocks([kc], [vc], torch.tensor([[src, dst]], dtype=torch.int32, device=device))
    torch.cuda.synchronize()
    assert torch.equal(kc[dst], kc[src]) and torch.equal(vc[dst], vc[src])
    if before is not None:
        assert torch.equal(kc[dst - 1], before)


def test_prefill_over_a_long_cached_prefix(device):
    """One sequence: 7168 cached tokens + 1024 new ones (128 KV tiles for the last chunk)."""
    rng = np.random.default_rng(23)
    L, P = 8192, 7168
    pages = L // 16
    ids = rng.permutation(pages + 7).astype(np.int32)[:pages]
    g = torch.Generator(device=device).manual_seed(23)
    kc = torch.randn((pages + 7, 8, 16, 128), device=device, generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    S = L - P
    q = torch.randn((S, 32, 128), device=device, generator=g).to(torch.bfloat16)
    bt = torch.from_numpy(ids.reshape(1, -1)).to(device)
    cu = torch.tensor([0, S], dtype=torch.int32, device=device)
    ctx = torch.tensor([L], dtype=torch.int32, device=device)
    scale = 1 / math.sqrt(128)
    out = ops.paged_prefill(q, kc, vc, cu, ctx, bt, 4, scale, S, L, ops.Workspace(device))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = oracle_attention(q, kc, vc, cu, ctx, bt, 4, scale)
    assert max_abs(f32(out), want) <= TOL
