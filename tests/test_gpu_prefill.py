"""Paged attention with several query tokens per sequence (prefill over cached prefixes).

* The reference's own attention tests (src/backend/cpu.rs:190-261) run on the GPU through the
  reference-shaped mirror ``paged_attention(q, blocks, n_rep, scale)``, same shapes and 1e-4.
* The float64 golden fixtures run through the GPU at 1e-4 (f32 pools).
* C3-shaped varlen prefill with shared prefix blocks, bf16, against the oracle at 2e-2.
"""

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from flour_b200 import ops
from flour_b200.paged import KvCache, SequenceBlocks, paged_attention
from flour_b200.workloads import LLAMA8B, Heads, make_c3

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def blocks_from_dense(k, v, block_size, device, seed=0):
    """(Hkv, kv, d) numpy -> a pool with shuffled physical blocks + the sequence's block list."""
    hkv, kv, d = k.shape
    nlog = -(-kv // block_size)
    nb = nlog + 2
    ids = np.random.default_rng(seed).permutation(nb)[:nlog]
    kc = np.zeros((nb, hkv, block_size, d), np.float32)
    vc = np.zeros_like(kc)
    for b in range(nlog):
        n = min(block_size, kv - b * block_size)
        kc[ids[b], :, :n] = k[:, b * block_size:b * block_size + n]
        vc[ids[b], :, :n] = v[:, b * block_size:b * block_size + n]
    return SequenceBlocks(torch.from_numpy(kc).to(device), torch.from_numpy(vc).to(device),
                          [int(i) for i in ids], kv)


def dense_ref(q, k, v, n_rep, scale):
    sq, kv = q.shape[1], k.shape[1]
    mask = (np.arange(kv)[None, :] > np.arange(sq)[:, None] + (kv - sq)).astype(np.uint8)
    return oracle.causal_attention(q, k, v, mask, scale, n_rep=n_rep)


@pytest.mark.parametrize("h,hkv,sq,kv,bs,seeds", [
    (2, 2, 5, 5, 2, (1, 2, 3)),     # paged_attention_matches_dense_prefill     cpu.rs:190-206
    (2, 2, 1, 7, 3, (10, 11, 12)),  # paged_attention_matches_dense_decode_step cpu.rs:208-224
    (4, 2, 6, 6, 4, (20, 21, 22)),  # paged_attention_matches_dense_with_gqa    cpu.rs:226-242
])
def test_reference_paged_vs_dense_on_gpu(device, h, hkv, sq, kv, bs, seeds):
    rngs = [np.random.default_rng(s) for s in seeds]
    q = rngs[0].uniform(-1, 1, (h, sq, 4)).astype(np.float32)
    k = rngs[1].uniform(-1, 1, (hkv, kv, 4)).astype(np.float32)
    v = rngs[2].uniform(-1, 1, (hkv, kv, 4)).astype(np.float32)
    scale = 1.0 / math.sqrt(4.0)
    ref = dense_ref(q, k, v, h // hkv, scale)
    out = paged_attention(torch.from_numpy(q)[None].to(device), blocks_from_dense(k, v, bs, device),
                          h // hkv, scale)
    assert tuple(out.shape) == (1, h, sq, 4)
    assert max_abs(f32(out[0]), ref) < 1e-4
    assert ops.device_status() == 0


def test_known_answer_on_gpu(device):  # cpu.rs:245-261
    lit = json.loads((GOLDEN / "reference_literals.json").read_text())["causal_known_answer"]
    q = torch.tensor(lit["q"], device=device).reshape(1, 1, 2, 1)
    k = np.array(lit["k"], np.float32).reshape(1, 2, 1)
    v = np.array(lit["v"], np.float32).reshape(1, 2, 1)
    out = paged_attention(q, blocks_from_dense(k, v, 1, device), 1, lit["scale"])
    np.testing.assert_allclose(f32(out).ravel(), lit["expected"], atol=lit["tol"])


@pytest.mark.parametrize("case", ["ref_prefill", "ref_decode", "ref_gqa", "c1_decode",
                                  "c1_prefix_prefill", "llama_decode"])
def test_golden_fixtures_on_gpu(device, case):
    z = np.load(GOLDEN / "dense_f64_cases.npz")
    q, k, v, want = (z[f"{case}/{x}"] for x in ("q", "k", "v", "out"))
    n_rep, scale, bs = int(z[f"{case}/n_rep"]), float(z[f"{case}/scale"]), int(z[f"{case}/block_size"])
    out = paged_attention(torch.from_numpy(q)[None].to(device), blocks_from_dense(k, v, bs, device, 5),
                          n_rep, scale)
    assert max_abs(f32(out[0]), want) < 1e-4


def small_c3(device, seed, dtype=torch.bfloat16, heads=LLAMA8B, n=8, lo=20, hi=300):
    return make_c3(device, seed=seed, dtype=dtype, heads=heads, num_seqs=n, group=4, lo=lo, hi=hi)


def run_prefill(b, write=True):
    h = b.heads
    if write:
        ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    return ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                             b.block_tables, h.n_rep, 1 / math.sqrt(h.head_dim), b.max_seqlen_q,
                             b.max_context_len, ops.Workspace(b.q.device))


@pytest.mark.parametrize("seed", [31, 32])
def test_c3_shaped_prefill_with_prefix_cache(device, seed):
    b = small_c3(device, seed)
    out = run_prefill(b)
    want = oracle_attention(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                            b.block_tables, b.heads.n_rep, 1 / math.sqrt(128))
    assert max_abs(f32(out), want) <= 2e-2
    assert ops.device_status() == 0


def test_prefill_f32_qwen_heads(device):
    b = small_c3(device, 33, dtype=torch.float32, heads=Heads(14, 2, 64), n=4, lo=17, hi=90)
    out = run_prefill(b)
    want = oracle_attention(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                            b.block_tables, 7, 1 / 8.0)
    assert max_abs(f32(out), want) <= 1e-5


def test_kv_cache_mirror_prefill_then_suffix(device):
    # Cold prefill of 40 tokens vs. prefix-reused suffix prefill over the same cache: the last
    # rows must agree (the invariance model.rs:244-360 checks at 1e-4, here f32).
    torch.manual_seed(1)
    hq, hkv, d = 4, 2, 16
    cache = KvCache(1, 64, hkv, d, torch.float32, device)
    k = torch.randn((1, hkv, 40, d), device=device)
    v = torch.randn((1, hkv, 40, d), device=device)
    q = torch.randn((1, hq, 40, d), device=device)
    cache.allocate_kv(40)
    cache.write_kv(0, k, v)
    cold = paged_attention(q, cache.kv_blocks(0), 2, 0.25)
    warm = paged_attention(q[:, :, 32:], cache.kv_blocks(0), 2, 0.25)
    assert max_abs(f32(cold[:, :, 32:]), f32(warm)) < 1e-5
