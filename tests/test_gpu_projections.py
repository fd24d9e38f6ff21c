"""The fused projections either side of attention against the oracle (oracle/projections.py,
restating src/models/common/attention.rs:75-116 and transformer.rs:37-38):

* fa_qkv_rope_cache: q/k/v projection (+ bias) -> per-head RMSNorm -> rotate-half RoPE ->
  q written token-major, k/v scattered into the paged pool by slot_mapping;
* fa_o_proj_residual: residual + attn W_o^T, checked against a plain PyTorch fp32 reference.

The kernels accumulate in f32 and round each output once, so the bar is the 16-bit rounding of
the result: |gpu - ref| <= 2e-3 + 8e-3 |ref| against the f32-flow oracle. The reference's own
dtype flow (a rounding after every op) is checked at 3e-2 + 2e-2 |ref|."""

import math

import numpy as np
import pytest
import torch

from flour_b200 import _lib, ops
from flour_b200.paged import rope_tables
from oracle import projections as P

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 8e-3


def close(got, want, atol=ATOL, rtol=RTOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want) - (atol + rtol * np.abs(want))
    assert err.max() <= 0, f"worst excess {err.max()} (max-abs {np.abs(got - want).max()})"


def f64(t):
    return t.detach().double().cpu().numpy()


def make_qkv(device, T, hidden, Hq, Hkv, d, dtype=torch.bfloat16, bias=False, qk_norm=False,
             seed=0, max_pos=4096, num_blocks=None, skip_every=0):
    g = torch.Generator().manual_seed(seed)
    N = (Hq + 2 * Hkv) * d
    x = torch.randn(T, hidden, generator=g).to(dtype)
    w = (torch.randn(N, hidden, generator=g) / math.sqrt(hidden)).to(dtype)
    b = (torch.randn(N, generator=g) * 0.2).to(dtype) if bias else None
    qn = (1 + 0.2 * torch.randn(d, generator=g)).to(dtype) if qk_norm else None
    kn = (1 + 0.2 * torch.randn(d, generator=g)).to(dtype) if qk_norm else None
    pos = torch.randint(0, max_pos, (T,), generator=g, dtype=torch.int32)
    bs = 16
    nb = num_blocks or (T // bs + 8)
    slots = torch.randperm(nb * bs, generator=g)[:T].to(torch.int32)
    if skip_every:
        slots[::skip_every] = -1
    kc = torch.randn(nb, Hkv, bs, d, generator=g).to(dtype)
    vc = torch.randn(nb, Hkv, bs, d, generator=g).to(dtype)
    cos, sin = rope_tables(d, max_pos, 10000.0, dtype)
    dev = lambda t: None if t is None else t.to(device)
    return dict(x=dev(x), w=dev(w), b=dev(b), qn=dev(qn), kn=dev(kn), pos=dev(pos),
                slots=dev(slots), kc=dev(kc), vc=dev(vc), cos=dev(cos), sin=dev(sin),
                Hq=Hq, Hkv=Hkv, d=d, bs=bs)


def run_qkv(c, eps=1e-6):
    kc0, vc0 = c["kc"].clone(), c["vc"].clone()
    q = ops.qkv_rope_cache(c["x"], c["w"], c["kc"], c["vc"], c["pos"], c["slots"], c["Hq"],
                           c["cos"], c["sin"], bias=c["b"], q_norm_weight=c["qn"],
                           k_norm_weight=c["kn"], rms_eps=eps)
    torch.cuda.synchronize()
    return q, kc0, vc0


def check_qkv(c, q, kc0, vc0, eps=1e-6):
    dt = "bf16" if c["x"].dtype == torch.bfloat16 else "f16"
    args = (f64(c["x"]), f64(c["w"]), c["Hq"], c["Hkv"], c["d"], c["pos"].cpu().numpy(),
            f64(c["cos"]), f64(c["sin"]), None if c["b"] is None else f64(c["b"]),
            None if c["qn"] is None else f64(c["qn"]), None if c["kn"] is None else f64(c["kn"]),
            eps)
    q_ref, k_ref, v_ref = P.qkv_forward(*args, flow="f32", dtype=dt)
    close(f64(q), q_ref)
    slots = c["slots"].cpu().numpy()
    live = np.nonzero(slots >= 0)[0]
    blk, off = slots[live] // c["bs"], slots[live] % c["bs"]
    kc, vc = f64(c["kc"]), f64(c["vc"])
    close(kc[blk, :, off, :], k_ref[live])
    close(vc[blk, :, off, :], v_ref[live])
    # every other pool row is untouched
    mask = np.ones(kc.shape[0] * c["bs"], bool)
    mask[slots[live]] = False
    untouched = np.nonzero(mask)[0]
    for cache, before in ((kc, f64(kc0)), (vc, f64(vc0))):
        a = cache.transpose(0, 2, 1, 3).reshape(-1, c["Hkv"], c["d"])[untouched]
        b = before.transpose(0, 2, 1, 3).reshape(-1, c["Hkv"], c["d"])[untouched]
        assert np.array_equal(a, b)
    # the reference's dtype flow, looser
    qc, kcand, _ = P.qkv_forward(*args, flow="candle", dtype=dt)
    close(f64(q), qc, 3e-2, 2e-2)
    close(kc[blk, :, off, :], kcand[live], 3e-2, 2e-2)


@pytest.mark.parametrize("T", [1, 64, 129, 300])
def test_qkv_llama_heads(device, T):
    c = make_qkv(device, T, 512, 8, 2, 128, seed=T)
    check_qkv(c, *run_qkv(c))
    assert ops.device_status() == 0


def test_qkv_bias_and_qk_norm(device):
    c = make_qkv(device, 200, 256, 4, 2, 128, bias=True, qk_norm=True, seed=5)
    check_qkv(c, *run_qkv(c, 1e-5), eps=1e-5)


def test_qkv_qwen05_heads_d64_f16_with_skips(device):
    # Qwen2.5-0.5B: hidden 896, 14 q heads, 2 kv heads, head_dim 64, qkv bias
    c = make_qkv(device, 333, 896, 14, 2, 64, dtype=torch.float16, bias=True, seed=6, skip_every=7)
    check_qkv(c, *run_qkv(c))


def test_qkv_k_not_multiple_of_64(device):
    c = make_qkv(device, 70, 520, 4, 1, 128, seed=7)
    check_qkv(c, *run_qkv(c))


def test_qkv_wide_grid_partial_n_tile(device):
    # enough tokens for 256-column tiles; (14 + 4) * 64 = 1152 columns leave a half tile
    c = make_qkv(device, 8192, 896, 14, 2, 64, bias=True, seed=8)
    check_qkv(c, *run_qkv(c))


def test_qkv_llama8b_shape(device):
    c = make_qkv(device, 1000, 4096, 32, 8, 128, seed=9)
    check_qkv(c, *run_qkv(c))


def test_qkv_bad_slot_and_position_are_reported_and_skipped(device):
    c = make_qkv(device, 64, 256, 4, 2, 128, seed=10, max_pos=128)
    nb = c["kc"].shape[0]
    c["slots"][3] = nb * 16 + 5      # past the pool
    c["pos"][5] = 128                # past the tables
    ops.device_status()
    q, kc0, vc0 = run_qkv(c)
    st = ops.device_status()
    assert st & _lib.FA_DEVERR_SLOT and st & _lib.FA_DEVERR_POSITION
    # rows with good data are still right
    good = [i for i in range(64) if i not in (3, 5)]
    dt = "bf16"
    q_ref, k_ref, v_ref = P.qkv_forward(f64(c["x"]), f64(c["w"]), 4, 2, 128,
                                        np.clip(c["pos"].cpu().numpy(), 0, 127), f64(c["cos"]),
                                        f64(c["sin"]), flow="f32", dtype=dt)
    close(f64(q)[good], q_ref[good])


def test_qkv_rejects_bad_arguments(device):
    c = make_qkv(device, 8, 64, 4, 2, 128)
    with pytest.raises(_lib.FlourAttnError):
        ops.qkv_rope_cache(c["x"], c["w"][:-1], c["kc"], c["vc"], c["pos"], c["slots"], 4,
                           c["cos"], c["sin"])
    kc32 = c["kc"].float()
    with pytest.raises(_lib.FlourAttnError) as e:
        ops.qkv_rope_cache(c["x"].float(), c["w"].float(), kc32, kc32.clone(), c["pos"], c["slots"],
                           4, c["cos"], c["sin"])
    assert e.value.status == _lib.FA_EUNSUPPORTED


@pytest.mark.parametrize("T,fin,fout", [(1, 4096, 4096), (64, 4096, 4096), (65, 4096, 4096),
                                        (300, 4096, 4096), (129, 896, 896),
                                        (8192, 896, 896), (2000, 3584, 3584)])
def test_o_proj_residual_vs_torch_fp32(device, T, fin, fout):
    g = torch.Generator(device=device).manual_seed(T + fin)
    a = torch.randn(T, fin, device=device, generator=g).to(torch.bfloat16)
    w = (torch.randn(fout, fin, device=device, generator=g) / math.sqrt(fin)).to(torch.bfloat16)
    r = torch.randn(T, fout, device=device, generator=g).to(torch.bfloat16)
    out = ops.o_proj_residual(a, w, r)
    want = r.float() + a.float() @ w.float().t()
    close(f64(out), f64(want))
    plain = ops.o_proj_residual(a, w)
    close(f64(plain), f64(a.float() @ w.float().t()))


def test_o_proj_residual_in_place_f16(device):
    g = torch.Generator(device=device).manual_seed(11)
    a = torch.randn(257, 1024, device=device, generator=g).half()
    w = (torch.randn(512, 1024, device=device, generator=g) / 32).half()
    h = torch.randn(257, 512, device=device, generator=g).half()
    want = h.float() + a.float() @ w.float().t()
    ops.o_proj_residual(a, w, h, out=h)   # residual aliases the output
    close(f64(h), f64(want))


def test_fused_layer_matches_unfused_path(device):
    """x -> fused QKV (+cache) -> paged prefill -> fused o_proj + residual equals the same layer
    built from the oracle pieces (the whole of CausalSelfAttention::forward + the residual)."""
    import oracle
    T, hidden, Hq, Hkv, d = 96, 512, 8, 2, 128
    c = make_qkv(device, T, hidden, Hq, Hkv, d, seed=12, num_blocks=16)
    # one sequence of T tokens at positions 0..T-1 in blocks 0..5
    c["pos"] = torch.arange(T, dtype=torch.int32, device=device)
    c["slots"] = torch.arange(T, dtype=torch.int32, device=device)
    q, _, _ = run_qkv(c)
    bt = torch.arange(16, dtype=torch.int32, device=device).reshape(1, 16)
    cu = torch.tensor([0, T], dtype=torch.int32, device=device)
    ctx = torch.tensor([T], dtype=torch.int32, device=device)
    scale = 1 / math.sqrt(d)
    attn = ops.paged_attention_varlen(q, c["kc"], c["vc"], cu, ctx, bt, Hq // Hkv, scale, T, T,
                                      ops.Workspace(device))
    g = torch.Generator(device=device).manual_seed(13)
    wo = (torch.randn(hidden, Hq * d, device=device, generator=g) / math.sqrt(Hq * d)).to(torch.bfloat16)
    out = ops.o_proj_residual(attn.reshape(T, Hq * d), wo, c["x"])
    # oracle path: same q/k/v (from the oracle), dense causal attention, projection + residual
    q_ref, k_ref, v_ref = P.qkv_forward(f64(c["x"]), f64(c["w"]), Hq, Hkv, d, np.arange(T),
                                        f64(c["cos"]), f64(c["sin"]))
    kk = np.repeat(k_ref, Hq // Hkv, axis=1)
    vv = np.repeat(v_ref, Hq // Hkv, axis=1)
    s = np.einsum("thd,jhd->htj", q_ref, kk) * scale
    s = s + np.triu(np.full((T, T), -np.inf), 1)[None]
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    y = np.einsum("htj,jhd->thd", p, vv).reshape(T, Hq * d)
    want = P.o_proj_residual(y, f64(wo), f64(c["x"]))
    got = f64(out)
    assert np.abs(got - want).max() <= 5e-2, np.abs(got - want).max()


# ---- fa_last_token_logits: final RMSNorm + lm_head on each sequence's last token ------------

def make_logits_case(device, lens, H, V, dtype, seed, norm=True):
    g = torch.Generator().manual_seed(seed)
    T = int(sum(lens))
    hidden = (torch.randn((T, H), generator=g) * 2.0).to(dtype).to(device)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(dtype).to(device) if norm else None
    lm = (torch.randn((V, H), generator=g) / math.sqrt(H)).to(dtype).to(device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    return hidden, w, lm, cu


@pytest.mark.parametrize("lens,H,V,dtype", [
    ([5, 1, 34, 1], 512, 1024, torch.bfloat16),
    ([3] * 200, 256, 2048, torch.bfloat16),      # 200 sequences: two 128-row M tiles
    ([64] * 8, 1024, 4096, torch.float16),
])
def test_last_token_logits_vs_oracle(device, lens, H, V, dtype):
    hidden, w, lm, cu = make_logits_case(device, lens, H, V, dtype, seed=len(lens) + H)
    logits = ops.last_token_logits(hidden, cu, lm, w, 1e-5)
    # The engine's readback: f32 rows into pinned host memory on the same stream.
    host = torch.empty(logits.shape, dtype=torch.float32, pin_memory=True)
    host.copy_(logits, non_blocking=True)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    dt = "bf16" if dtype == torch.bfloat16 else "f16"
    args = (f64(hidden), cu.cpu().numpy(), None if w is None else f64(w), f64(lm), 1e-5)
    # Kernel flow: the norm rounded once to the model dtype (the GEMM operand), logits in f32.
    close(host.numpy(), P.last_token_logits(*args, flow="f32", dtype=dt, norm_flow="candle"))
    # The reference's own flow rounds the norm and the logits to the model dtype.
    close(host.numpy(), P.last_token_logits(*args, flow="candle", dtype=dt), 3e-2, 2e-2)


def test_last_token_logits_no_norm_weight_and_bad_sequence(device):
    hidden, _, lm, cu = make_logits_case(device, [7, 9, 4], 256, 512, torch.bfloat16, 3, norm=False)
    ops.device_status()
    logits = ops.last_token_logits(hidden, cu, lm, None, 1e-6)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    close(f64(logits), P.last_token_logits(f64(hidden), cu.cpu().numpy(), None, f64(lm), 1e-6,
                                           dtype="bf16", norm_flow="candle"))
    bad = cu.clone()
    bad[2] = bad[1]  # sequence 1 empty: zero logits and FA_DEVERR_SEQLEN, the others intact
    logits2 = ops.last_token_logits(hidden, bad, lm, None, 1e-6)
    torch.cuda.synchronize()
    assert ops.device_status() & _lib.FA_DEVERR_SEQLEN
    assert not logits2[1].any()
    assert torch.equal(logits2[2], logits[2])


def test_last_token_logits_rejects_bad_arguments(device):
    hidden, w, lm, cu = make_logits_case(device, [4, 4], 256, 512, torch.bfloat16, 4)
    with pytest.raises(_lib.FlourAttnError):
        ops.last_token_logits(hidden, cu, lm[:500], w)        # vocab not a multiple of 32
    with pytest.raises(_lib.FlourAttnError):
        ops.last_token_logits(hidden.float(), cu, lm, w)      # f32 hidden


def test_gemm_tile_width_query(device):
    L = _lib.lib()
    # The C2 lm_head (64 rows, 128256 columns): 128-column tiles (7 waves of 128 columns on the
    # busiest SM instead of 4 of 256). A C3-sized QKV projection fills the GPU with 256-wide
    # tiles; a decode-batch QKV splits K over a cluster (128-wide tiles).
    assert L.fa_gemm_tile_width(64, 128256, 4096) == 128
    assert L.fa_gemm_tile_width(15401, 6144, 4096) == 256
    assert L.fa_gemm_tile_width(64, 6144, 4096) == 128
    assert L.fa_gemm_tile_width(0, 6144, 4096) == 0
