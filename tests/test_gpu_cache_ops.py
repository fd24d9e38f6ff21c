"""Block writes and block copies on the GPU, bit-exact against the oracle, plus the reference's
pool tests (src/models/common/paged.rs:287-340) through the PagedKvPool mirror."""

import numpy as np
import pytest
import torch

import oracle
from flour_b200 import FlourAttnError, _lib, ops
from flour_b200.paged import KvCache, PagedKvPool
from flour_b200.workloads import to_numpy

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def rand(shape, dtype, device, gen):
    return torch.randn(shape, device=device, generator=gen).to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("nb,kvh,bs,d", [(64, 8, 16, 128), (40, 2, 16, 64), (9, 3, 2, 4),
                                         (16, 1, 5, 6)])
def test_reshape_and_cache_bit_exact(device, dtype, nb, kvh, bs, d):
    gen = torch.Generator(device=device).manual_seed(nb * 7 + d)
    kc = rand((nb, kvh, bs, d), dtype, device, gen)
    vc = rand((nb, kvh, bs, d), dtype, device, gen)
    T = min(nb * bs, 300)
    rng = np.random.default_rng(d)
    slots = rng.permutation(nb * bs)[:T].astype(np.int32)
    slots[::7] = -1  # skipped tokens
    key = rand((T, kvh, d), dtype, device, gen)
    value = rand((T, kvh, d), dtype, device, gen)
    want_k, want_v = to_numpy(kc), to_numpy(vc)
    assert oracle.reshape_and_cache(want_k, want_v, to_numpy(key), to_numpy(value), slots) == 0
    ops.reshape_and_cache(kc, vc, key, value, torch.from_numpy(slots).to(device))
    assert ops.device_status() == 0
    np.testing.assert_array_equal(to_numpy(kc), want_k)
    np.testing.assert_array_equal(to_numpy(vc), want_v)


def test_reshape_and_cache_heads_major_strides(device):
    # The reference hands k as (1, kv_heads, n, d) (attention.rs:92-104): pass it as a strided view.
    gen = torch.Generator(device=device).manual_seed(3)
    nb, kvh, bs, d, n = 32, 4, 16, 128, 37
    kc = torch.zeros((nb, kvh, bs, d), dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    k = rand((1, kvh, n, d), torch.bfloat16, device, gen)
    v = rand((1, kvh, n, d), torch.bfloat16, device, gen)
    slots = np.random.default_rng(1).permutation(nb * bs)[:n].astype(np.int32)
    ops.reshape_and_cache(kc, vc, k[0].transpose(0, 1), v[0].transpose(0, 1),
                          torch.from_numpy(slots).to(device))
    want_k, want_v = np.zeros_like(to_numpy(kc)), np.zeros_like(to_numpy(vc))
    oracle.reshape_and_cache(want_k, want_v, to_numpy(k[0].transpose(0, 1)),
                             to_numpy(v[0].transpose(0, 1)), slots)
    np.testing.assert_array_equal(to_numpy(kc), want_k)
    np.testing.assert_array_equal(to_numpy(vc), want_v)


def test_reshape_and_cache_reports_out_of_range_slot(device):
    kc = torch.zeros((4, 1, 2, 8), dtype=torch.float32, device=device)
    vc = torch.zeros_like(kc)
    key = torch.ones((3, 1, 8), device=device)
    ops.device_status()
    ops.reshape_and_cache(kc, vc, key, key, torch.tensor([1, 8, -1], dtype=torch.int32, device=device))
    assert ops.device_status() == _lib.FA_DEVERR_SLOT
    assert kc[0, 0, 1].tolist() == [1.0] * 8 and float(kc.sum()) == 8.0


@pytest.mark.parametrize("dtype", DTYPES)
def test_copy_blocks_bit_exact(device, dtype):
    gen = torch.Generator(device=device).manual_seed(11)
    L, nb, kvh, bs, d = 3, 50, 8, 16, 128
    kcs = [rand((nb, kvh, bs, d), dtype, device, gen) for _ in range(L)]
    vcs = [rand((nb, kvh, bs, d), dtype, device, gen) for _ in range(L)]
    rng = np.random.default_rng(2)
    perm = rng.permutation(nb)
    pairs = np.stack([perm[:12], perm[12:24]], axis=1).astype(np.int32)  # disjoint src/dst
    wk, wv = [to_numpy(x) for x in kcs], [to_numpy(x) for x in vcs]
    assert oracle.copy_blocks(wk, wv, pairs) == 0
    ops.copy_blocks(kcs, vcs, torch.from_numpy(pairs).to(device))
    assert ops.device_status() == 0
    for l in range(L):
        np.testing.assert_array_equal(to_numpy(kcs[l]), wk[l])
        np.testing.assert_array_equal(to_numpy(vcs[l]), wv[l])


def test_copy_blocks_reports_bad_pair(device):
    kc = torch.arange(4 * 2 * 4, dtype=torch.float32, device=device).reshape(4, 1, 2, 4)
    vc = kc.clone()
    before = kc.clone()
    ops.device_status()
    ops.copy_blocks([kc], [vc], torch.tensor([[0, 7], [1, 2]], dtype=torch.int32, device=device))
    assert ops.device_status() == _lib.FA_DEVERR_PAIR
    assert torch.equal(kc[2], before[1]) and torch.equal(kc[3], before[3])


def test_pool_write_then_gather_round_trips(device):  # paged.rs:287-306
    pool = PagedKvPool(1, 2, 1, 2, torch.float32, device, block_size=2)
    k = torch.tensor([1.0, 2.0, 3.0, 4.0], device=device).reshape(1, 1, 2, 2)
    v = torch.tensor([5.0, 6.0, 7.0, 8.0], device=device).reshape(1, 1, 2, 2)
    pool.write(0, [2, 0], k, v)
    gk, gv = pool.gather(0, [0, 2])
    assert tuple(gk.shape) == (1, 1, 2, 2)
    assert gk.flatten().tolist() == [3.0, 4.0, 1.0, 2.0]
    assert gv.flatten().tolist() == [7.0, 8.0, 5.0, 6.0]


def test_pool_write_block_round_trips_full_block(device):  # paged.rs:309-331
    pool = PagedKvPool(1, 2, 1, 2, torch.float32, device, block_size=2)
    k = torch.tensor([1.0, 2.0, 3.0, 4.0]).reshape(1, 1, 2, 2)  # host tensor: H2D copy
    v = torch.tensor([5.0, 6.0, 7.0, 8.0]).reshape(1, 1, 2, 2)
    pool.write_block(0, 1, k, v)
    torch.cuda.synchronize()
    rk, rv = pool.block_view(0, 2, 2)
    assert tuple(rk.shape) == (1, 1, 2, 2)
    assert rk.flatten().tolist() == [1.0, 2.0, 3.0, 4.0]
    assert rv.flatten().tolist() == [5.0, 6.0, 7.0, 8.0]
    zk, _ = pool.block_view(0, 0, 2)
    assert zk.flatten().tolist() == [0.0] * 4


def test_write_block_rejects_mismatched_kv_heads(device):  # paged.rs:333-340
    pool = PagedKvPool(1, 2, 1, 2, torch.float32, device, block_size=2)
    k = torch.zeros((1, 2, 2, 2), device=device)
    with pytest.raises(ValueError):
        pool.write_block(0, 0, k, k)


def test_write_and_read_block_host_round_trip(device):
    nb, kvh, bs, d = 6, 8, 16, 128
    kc = torch.zeros((nb, kvh, bs, d), dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    k = torch.randn((kvh, bs, d)).to(torch.bfloat16).pin_memory()
    v = torch.randn((kvh, bs, d)).to(torch.bfloat16).pin_memory()
    ops.write_block(kc, vc, 4, k, v)
    ko = torch.empty_like(k).pin_memory()
    vo = torch.empty_like(v).pin_memory()
    ops.read_block(kc, vc, 4, ko, vo)
    torch.cuda.synchronize()
    assert torch.equal(ko, k) and torch.equal(vo, v)
    assert float(kc[:4].abs().sum()) == 0.0 and float(kc[5].abs().sum()) == 0.0
    with pytest.raises(FlourAttnError):
        ops.write_block(kc, vc, nb, k, v)


def test_bundle_export_payload_order_through_read_block(device):
    # KvCache::export_prefix_bundle (cache.rs:166-228): block-major, then layer, then K, V.
    L, kvh, d = 2, 2, 4
    cache = KvCache(L, 64, kvh, d, torch.float32, device)
    cache.allocate_kv(32)
    for layer in range(L):  # cache.rs:740-752 values
        n = kvh * 32 * d
        kd = (layer * 1000 + torch.arange(n, dtype=torch.float32)).reshape(1, kvh, 32, d).to(device)
        cache.write_kv(layer, kd, kd + 0.25)
    blocks = cache.table.blocks()
    pieces = []
    for b in blocks:
        for layer in range(L):
            ko = torch.empty((kvh, 16, d))
            vo = torch.empty((kvh, 16, d))
            ops.read_block(cache.pool.k_pools[layer], cache.pool.v_pools[layer], b, ko, vo)
            torch.cuda.synchronize()
            pieces += [ko.numpy().ravel(), vo.numpy().ravel()]
    payload = np.concatenate(pieces).view(np.uint8)
    want = oracle.bundle_export([to_numpy(x) for x in cache.pool.k_pools],
                                [to_numpy(x) for x in cache.pool.v_pools], blocks)
    np.testing.assert_array_equal(payload, want)


def _bundle_pools(device, layers, nb, kvh, d, dtype, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    ks = [torch.randn((nb, kvh, 16, d), device=device, generator=g).to(dtype) for _ in range(layers)]
    vs = [torch.randn((nb, kvh, 16, d), device=device, generator=g).to(dtype) for _ in range(layers)]
    return ks, vs


def test_bundle_payload_export_one_launch_matches_oracle(device):
    # A 2048-token prefix of Llama-3-8B: 128 blocks x 32 layers, gathered in one launch into the
    # FLKV payload order (bundle.rs:15-22), bit-exact against the oracle's restatement.
    L, nb = 32, 512
    ks, vs = _bundle_pools(device, L, nb, 8, 128, torch.bfloat16, 40)
    ids = torch.from_numpy(np.random.default_rng(40).permutation(nb)[:128].astype(np.int32)).to(device)
    payload = ops.export_bundle_payload(ks, vs, ids)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert payload.numel() == 128 * L * 2 * 8 * 16 * 128 * 2
    want = oracle.bundle_export([to_numpy(x) for x in ks], [to_numpy(x) for x in vs],
                                ids.cpu().numpy())
    np.testing.assert_array_equal(payload.cpu().numpy(), want)


@pytest.mark.parametrize("dtype,kvh,d", [(torch.float32, 2, 64), (torch.float16, 4, 128),
                                         (torch.bfloat16, 1, 96)])
def test_bundle_payload_round_trip_and_neighbours(device, dtype, kvh, d):
    # Export from one pool, import into other physical blocks of a second pool (the importing
    # node's own allocation): bit-exact against the oracle import, every other block untouched.
    L, nb, n = 3, 40, 7
    ks, vs = _bundle_pools(device, L, nb, kvh, d, dtype, 41)
    src = torch.tensor([5, 0, 39, 12, 7, 8, 21], dtype=torch.int32, device=device)
    payload = ops.export_bundle_payload(ks, vs, src)
    k2, v2 = _bundle_pools(device, L, nb, kvh, d, dtype, 42)
    k2_np, v2_np = [to_numpy(x) for x in k2], [to_numpy(x) for x in v2]
    dst = torch.tensor([30, 31, 1, 2, 17, 18, 3], dtype=torch.int32, device=device)
    ops.import_bundle_payload(k2, v2, dst, payload)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    oracle.bundle_import(k2_np, v2_np, dst.cpu().numpy(), payload.cpu().numpy())
    for l in range(L):
        np.testing.assert_array_equal(to_numpy(k2[l]), k2_np[l])
        np.testing.assert_array_equal(to_numpy(v2[l]), v2_np[l])
        assert torch.equal(k2[l][dst.long()], ks[l][src.long()])


def test_bundle_payload_bad_block_id(device):
    L, nb = 2, 8
    ks, vs = _bundle_pools(device, L, nb, 2, 64, torch.bfloat16, 43)
    ops.device_status()
    ids = torch.tensor([1, nb, 2], dtype=torch.int32, device=device)
    payload = ops.export_bundle_payload(ks, vs, ids)
    torch.cuda.synchronize()
    assert ops.device_status() & _lib.FA_DEVERR_BLOCK_ID
    piece = 2 * 16 * 64 * 2
    p = payload.view(3, L, 2, piece)
    assert int(p[1].abs().sum()) == 0  # the bad block's pieces are zero-filled
    assert torch.equal(p[0, 0, 0].view(torch.bfloat16).view(2, 16, 64), ks[0][1])
    before = [k.clone() for k in ks]
    ops.import_bundle_payload(ks, vs, ids, payload)
    torch.cuda.synchronize()
    assert ops.device_status() & _lib.FA_DEVERR_BLOCK_ID
    assert all(torch.equal(a, b) for a, b in zip(ks, before))  # same data back in blocks 1, 2
