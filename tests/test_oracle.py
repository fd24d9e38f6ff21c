"""The CPU oracle pinned against the reference's own tests and the golden fixtures.

Ports (same shapes, values and tolerances) of:
  src/backend/cpu.rs:119-137     repeat_kv shapes (as the GQA head mapping)
  src/backend/cpu.rs:190-242     paged_attention == dense causal_attention within 1e-4
  src/backend/cpu.rs:245-261     causal_attention known answer (10.0, 15.0)
  src/models/common/paged.rs:287-331, 378-394   pool write/gather/write_block/slot goldens
  src/models/common/cache.rs:727-783 / bundle.rs  bundle payload order
"""

import json
import zlib
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
LIT = json.loads((GOLDEN / "reference_literals.json").read_text())


def pool_from_dense(k, v, block_size, rng=None, extra_blocks=3):
    """Dense (Hkv, kv, d) -> build-layout pool with the logical blocks at shuffled physical ids."""
    hkv, kv, d = k.shape
    nlog = -(-kv // block_size)
    nb = nlog + extra_blocks
    ids = (rng.permutation(nb) if rng is not None else np.arange(nb))[:nlog].astype(np.int32)
    kc = np.full((nb, hkv, block_size, d), np.nan, dtype=np.float32)  # NaN canaries
    vc = np.full_like(kc, np.nan)
    for b in range(nlog):
        n = min(block_size, kv - b * block_size)
        kc[ids[b], :, :n] = k[:, b * block_size:b * block_size + n]
        vc[ids[b], :, :n] = v[:, b * block_size:b * block_size + n]
        kc[ids[b], :, n:] = 0.0
        vc[ids[b], :, n:] = 0.0
    return kc, vc, ids


def run_paged(q, k, v, n_rep, scale, block_size, rng=None, score_mode=0):
    """q (H, sq, d) one sequence -> (H, sq, d) through oracle.paged_attention."""
    h, sq, d = q.shape
    kc, vc, ids = pool_from_dense(k, v, block_size, rng)
    qp = np.ascontiguousarray(q.transpose(1, 0, 2))
    out, err = oracle.paged_attention(qp, kc, vc, [0, sq], [k.shape[1]], ids[None, :], n_rep,
                                      scale, score_mode=score_mode)
    assert err == 0
    return out.transpose(1, 0, 2)


def dense_ref(q, k, v, n_rep, scale):
    sq, kv = q.shape[1], k.shape[1]
    mask = (np.arange(kv)[None, :] > np.arange(sq)[:, None] + (kv - sq)).astype(np.uint8)
    return oracle.causal_attention(q, k, v, mask, scale, n_rep=n_rep)


def uniform(shape, rng):
    return rng.uniform(-1.0, 1.0, shape).astype(np.float32)


def test_gqa_head_mapping_matches_repeat_kv():
    # cpu.rs:5-13: expanding KV heads n_rep times == query head h reading kv head h / n_rep.
    rng = np.random.default_rng(0)
    q, k, v = uniform((6, 3, 4), rng), uniform((2, 3, 4), rng), uniform((2, 3, 4), rng)
    ke, ve = np.repeat(k, 3, axis=0), np.repeat(v, 3, axis=0)
    a = dense_ref(q, k, v, 3, 0.5)
    b = dense_ref(q, ke, ve, 1, 0.5)
    np.testing.assert_array_equal(a, b)
    assert ke.shape == (6, 3, 4)  # cpu.rs:129-137 shape


@pytest.mark.parametrize("name,h,hkv,sq,kv,bs", [
    ("prefill", 2, 2, 5, 5, 2),   # cpu.rs:190-206 (partial last block)
    ("decode", 2, 2, 1, 7, 3),    # cpu.rs:208-224
    ("gqa", 4, 2, 6, 6, 4),       # cpu.rs:226-242
])
def test_paged_matches_dense_reference_tests(name, h, hkv, sq, kv, bs):
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    q, k, v = uniform((h, sq, 4), rng), uniform((hkv, kv, 4), rng), uniform((hkv, kv, 4), rng)
    scale = 1.0 / np.sqrt(4.0)
    ref = dense_ref(q, k, v, h // hkv, scale)
    out = run_paged(q, k, v, h // hkv, scale, bs, rng)
    assert np.abs(out - ref).max() < 1e-4


def test_causal_known_answer():
    c = LIT["causal_known_answer"]
    q = np.array(c["q"], np.float32).reshape(1, 2, 1)
    k = np.array(c["k"], np.float32).reshape(1, 2, 1)
    v = np.array(c["v"], np.float32).reshape(1, 2, 1)
    out = oracle.causal_attention(q, k, v, np.array(c["mask"], np.uint8), c["scale"])
    np.testing.assert_allclose(out.ravel(), c["expected"], atol=c["tol"])


def test_paged_known_answer_through_blocks():
    # The same known answer through the paged fold with one-token blocks.
    c = LIT["causal_known_answer"]
    q = np.array(c["q"], np.float32).reshape(1, 2, 1)
    k = np.array(c["k"], np.float32).reshape(1, 2, 1)
    v = np.array(c["v"], np.float32).reshape(1, 2, 1)
    out = run_paged(q, k, v, 1, c["scale"], 1)
    np.testing.assert_allclose(out.ravel(), c["expected"], atol=c["tol"])


@pytest.mark.parametrize("case", ["ref_prefill", "ref_decode", "ref_gqa", "c1_decode",
                                  "c1_prefix_prefill", "llama_decode"])
def test_oracle_against_float64_golden(case):
    z = np.load(GOLDEN / "dense_f64_cases.npz")
    q, k, v, want = (z[f"{case}/{x}"] for x in ("q", "k", "v", "out"))
    n_rep, scale, bs = int(z[f"{case}/n_rep"]), float(z[f"{case}/scale"]), int(z[f"{case}/block_size"])
    out = run_paged(q, k, v, n_rep, scale, bs, np.random.default_rng(7))
    assert np.abs(out - want).max() < 1e-4  # the reference's paged-vs-dense tolerance
    dense = dense_ref(q, k, v, n_rep, scale)
    assert np.abs(dense - want).max() < 1e-4


def test_bf16_modes_agree_within_tolerance():
    # score_mode 1 (candle's dtype flow) and 0 (f32 scores) differ only by bf16 score rounding.
    rng = np.random.default_rng(11)
    q = oracle.f32_to_bf16(rng.standard_normal((32, 1, 128)).astype(np.float32))
    k = oracle.f32_to_bf16(rng.standard_normal((8, 300, 128)).astype(np.float32))
    v = oracle.f32_to_bf16(rng.standard_normal((8, 300, 128)).astype(np.float32))
    kc, vc, ids = pool_from_dense(oracle.bf16_to_f32(k), oracle.bf16_to_f32(v), 16, rng)
    kc, vc = oracle.f32_to_bf16(np.nan_to_num(kc)), oracle.f32_to_bf16(np.nan_to_num(vc))
    qp = np.ascontiguousarray(q.transpose(1, 0, 2))
    args = (qp, kc, vc, [0, 1], [300], ids[None, :], 4, 1 / np.sqrt(128))
    o0, _ = oracle.paged_attention(*args, dtype=oracle.DT_BF16, score_mode=0)
    o1, _ = oracle.paged_attention(*args, dtype=oracle.DT_BF16, score_mode=1)
    d = np.abs(oracle.bf16_to_f32(o0) - oracle.bf16_to_f32(o1)).max()
    assert d < 2e-2


def test_slot_mapping_golden():
    c = LIT["slot_mapping"]
    for pos, want in c["slot"].items():
        assert oracle.slot(c["blocks"], c["block_size"], int(pos)) == want
    assert list(oracle.slots(c["blocks"], c["block_size"], 0, 3)) == c["slots_0_3"]


def test_pool_write_then_gather_golden():
    c = LIT["write_then_gather"]
    kp = np.zeros((c["kv_heads"], c["num_slots"], c["head_dim"]), np.float32)
    vp = np.zeros_like(kp)
    k = np.array(c["k"], np.float32).reshape(1, 2, 2)
    v = np.array(c["v"], np.float32).reshape(1, 2, 2)
    assert oracle.pool_write_literal(kp, vp, c["slots"], k, v) == 0
    np.testing.assert_array_equal(kp[:, c["gather_slots"]].ravel(), c["gk"])
    np.testing.assert_array_equal(vp[:, c["gather_slots"]].ravel(), c["gv"])


def test_scatter_matches_literal_write_on_reference_case():
    # Same test through the build layout (bs=2): slots 2 and 0 -> blocks 1 and 0.
    c = LIT["write_then_gather"]
    kc = np.zeros((2, 1, 2, 2), np.float32)
    vc = np.zeros_like(kc)
    key = np.array(c["k"], np.float32).reshape(2, 1, 2)
    val = np.array(c["v"], np.float32).reshape(2, 1, 2)
    assert oracle.reshape_and_cache(kc, vc, key, val, c["slots"]) == 0
    flat_k = kc.transpose(1, 0, 2, 3).reshape(1, 4, 2)
    flat_v = vc.transpose(1, 0, 2, 3).reshape(1, 4, 2)
    np.testing.assert_array_equal(flat_k[:, c["gather_slots"]].ravel(), c["gk"])
    np.testing.assert_array_equal(flat_v[:, c["gather_slots"]].ravel(), c["gv"])


def test_literal_write_run_condition_differs_from_per_slot_scatter():
    # paged.rs:196 tests `i + n == start_slot + n` (i.e. i == start_slot) instead of comparing
    # the next slot: when a token's batch index equals its slot, the run swallows every later
    # token. Slots [0, 5]: the reference writes token 1 to slot 1, a per-slot scatter to slot 5.
    kp_lit = np.zeros((1, 8, 2), np.float32)
    vp_lit = np.zeros_like(kp_lit)
    k = np.array([[[1, 2], [3, 4]]], np.float32)
    assert oracle.pool_write_literal(kp_lit, vp_lit, [0, 5], k, k) == 0
    assert kp_lit[0, 1].tolist() == [3, 4] and kp_lit[0, 5].tolist() == [0, 0]
    kc = np.zeros((4, 1, 2, 2), np.float32)
    assert oracle.reshape_and_cache(kc, kc.copy(), k.transpose(1, 0, 2), k.transpose(1, 0, 2),
                                    [0, 5]) == 0
    flat = kc.transpose(1, 0, 2, 3).reshape(1, 8, 2)
    assert flat[0, 5].tolist() == [3, 4] and flat[0, 1].tolist() == [0, 0]


def test_literal_write_equals_scatter_when_no_index_equals_its_slot():
    rng = np.random.default_rng(5)
    for _ in range(50):
        n = int(rng.integers(1, 20))
        slots = rng.permutation(64)[:n].astype(np.uint32)
        if np.any(slots == np.arange(n)):
            continue
        k = rng.standard_normal((2, n, 4)).astype(np.float32)
        kp = np.zeros((2, 64, 4), np.float32)
        oracle.pool_write_literal(kp, kp.copy(), slots, k, k)
        kc = np.zeros((16, 2, 4, 4), np.float32)
        oracle.reshape_and_cache(kc, kc.copy(), k.transpose(1, 0, 2), k.transpose(1, 0, 2), slots)
        np.testing.assert_array_equal(kc.transpose(1, 0, 2, 3).reshape(2, 64, 4), kp)


def test_write_block_round_trip_golden():
    c = LIT["write_block_round_trip"]
    kc = np.zeros((2, 1, 2, 2), np.float32)
    vc = np.zeros_like(kc)
    src_k = np.zeros_like(kc)
    src_v = np.zeros_like(kc)
    src_k[0] = np.array(c["k"], np.float32).reshape(1, 2, 2)
    src_v[0] = np.array(c["v"], np.float32).reshape(1, 2, 2)
    # write_block(block 1) == copy of a block holding those values into block 1.
    kk = np.concatenate([src_k[:1], kc[:1]])
    vv = np.concatenate([src_v[:1], vc[:1]])
    assert oracle.copy_blocks([kk], [vv], [[0, 1]]) == 0
    np.testing.assert_array_equal(kk[1].ravel(), c["k"])
    np.testing.assert_array_equal(vv[1].ravel(), c["v"])


def test_reshape_and_cache_reports_bad_slots():
    kc = np.zeros((2, 1, 2, 2), np.float32)
    key = np.ones((3, 1, 2), np.float32)
    err = oracle.reshape_and_cache(kc, kc.copy(), key, key, [-1, 4, 1])
    assert err == oracle.ERR_SLOT
    assert kc[0, 0, 1].tolist() == [1, 1] and kc.sum() == 2


def test_bundle_payload_order():
    c = LIT["bundle_export_values"]
    hkv, d, L, T, bs = c["kv_heads"], c["head_dim"], c["num_layers"], c["tokens"], c["block_size"]
    ids = np.array([3, 1], np.int32)  # logical blocks 0, 1 at physical 3, 1
    kcs, vcs = [], []
    for layer in range(L):
        kdense = (layer * 1000 + np.arange(hkv * T * d)).astype(np.float32).reshape(hkv, T, d)
        kc = np.zeros((4, hkv, bs, d), np.float32)
        for b in range(2):
            kc[ids[b]] = kdense[:, b * bs:(b + 1) * bs]
        kcs.append(kc)
        vcs.append(kc + c["v_offset"])
    payload = oracle.bundle_export(kcs, vcs, ids).view(np.float32)
    per = hkv * bs * d
    o = 0
    for b in range(2):
        for layer in range(L):
            kdense = (layer * 1000 + np.arange(hkv * T * d)).astype(np.float32).reshape(hkv, T, d)
            want = kdense[:, b * bs:(b + 1) * bs].ravel()
            np.testing.assert_array_equal(payload[o:o + per], want)
            np.testing.assert_array_equal(payload[o + per:o + 2 * per], want + c["v_offset"])
            o += 2 * per
    # Import into other physical blocks and read back the same payload.
    kcs2 = [np.zeros_like(x) for x in kcs]
    vcs2 = [np.zeros_like(x) for x in vcs]
    oracle.bundle_import(kcs2, vcs2, [0, 2], payload.view(np.uint8))
    np.testing.assert_array_equal(oracle.bundle_export(kcs2, vcs2, [0, 2]), payload.view(np.uint8))


def test_oracle_reports_bad_block_ids_and_context():
    kc = np.zeros((4, 1, 2, 2), np.float32)
    q = np.ones((2, 1, 2), np.float32)
    out, err = oracle.paged_attention(q, kc, kc, [0, 1, 2], [3, 3], [[0, 9], [0, 1]], 1, 1.0)
    assert err == oracle.ERR_BLOCK_ID
    out, err = oracle.paged_attention(q, kc, kc, [0, 1, 2], [5, 3], [[0, 1], [0, 1]], 1, 1.0)
    assert err == oracle.ERR_CONTEXT
