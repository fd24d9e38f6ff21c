"""Self-checks of the projection oracle (oracle/projections.py) on the CPU: the rotate-half RoPE
restatement of candle_nn::rotary_emb::rope (used at src/models/common/attention.rs:96-99), the
tables of Cache::new (src/models/common/cache.rs:378-392), bf16 rounding, and agreement between
the f32 flow and the reference's dtype flow."""

import numpy as np
import torch

from oracle import projections as P
from flour_b200.paged import rope_tables


def test_round_to_bf16_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 37.0
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(P.round_to(x, "bf16"), want.astype(np.float64))
    want16 = torch.from_numpy(x).to(torch.float16).float().numpy()
    assert np.array_equal(P.round_to(x, "f16"), want16.astype(np.float64))


def test_rope_tables_match_host_mirror():
    for d, dt, tdt in ((128, "bf16", torch.bfloat16), (64, "f16", torch.float16)):
        c, s = P.rope_tables(d, 4096, 10000.0, dt)
        tc, ts = rope_tables(d, 4096, 10000.0, tdt)
        # f32 angles from two libraries' pow/cos/sin may differ by an ulp before rounding.
        assert np.abs(c - tc.numpy()).max() <= 2 ** -7
        assert np.abs(s - ts.numpy()).max() <= 2 ** -7
        assert np.mean(c == tc.numpy()) > 0.99
    c, s = P.rope_tables(128, 8, 10000.0, "bf16")
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)  # position 0: no rotation


def test_rope_is_a_rotation_with_relative_positions():
    rng = np.random.default_rng(1)
    d = 128
    ang_theta = 1.0 / 10000.0 ** (np.arange(d // 2) * 2 / d)
    def tab(p):
        a = p * ang_theta
        return np.cos(a), np.sin(a)
    q, k = rng.standard_normal(d), rng.standard_normal(d)
    # pair norms preserved
    c, s = tab(37)
    rq = P.rope(q, c, s)
    h = d // 2
    assert np.allclose(rq[:h] ** 2 + rq[h:] ** 2, q[:h] ** 2 + q[h:] ** 2)
    # <rope(q, m), rope(k, n)> depends only on m - n
    dots = []
    for m, n in ((10, 3), (107, 100), (1007, 1000)):
        cm, sm = tab(m)
        cn, sn = tab(n)
        dots.append(P.rope(q, cm, sm) @ P.rope(k, cn, sn))
    assert np.allclose(dots, dots[0])
    # position 0 is the identity
    assert np.allclose(P.rope(q, np.ones(h), np.zeros(h)), q)


def test_qkv_flows_agree_within_bf16_rounding():
    rng = np.random.default_rng(2)
    T, hidden, Hq, Hkv, d = 9, 64, 4, 2, 16
    r = lambda a: P.round_to(a, "bf16")
    x = r(rng.standard_normal((T, hidden)))
    w = r(rng.standard_normal(((Hq + 2 * Hkv) * d, hidden)) / 8.0)
    b = r(rng.standard_normal((Hq + 2 * Hkv) * d) * 0.1)
    qn, kn = r(1 + 0.1 * rng.standard_normal(d)), r(1 + 0.1 * rng.standard_normal(d))
    cos, sin = P.rope_tables(d, 64, 10000.0, "bf16")
    pos = rng.integers(0, 64, size=T)
    a = P.qkv_forward(x, w, Hq, Hkv, d, pos, cos, sin, b, qn, kn, 1e-6, "f32")
    c = P.qkv_forward(x, w, Hq, Hkv, d, pos, cos, sin, b, qn, kn, 1e-6, "candle")
    for u, v in zip(a, c):
        assert np.abs(u - v).max() <= 3e-2 * max(1.0, np.abs(u).max())
    # v has no RoPE: it is the third slice of the projection
    y = x @ w.T + b
    assert np.allclose(a[2], y[:, (Hq + Hkv) * d:].reshape(T, Hkv, d))


def test_o_proj_residual_oracle():
    rng = np.random.default_rng(3)
    a, w, res = rng.standard_normal((5, 32)), rng.standard_normal((16, 32)), rng.standard_normal((5, 16))
    assert np.allclose(P.o_proj_residual(a, w, res), res + a @ w.T)
    assert np.allclose(P.o_proj_residual(a, w), a @ w.T)


def test_last_token_logits_oracle():
    # engine.rs:220-222 reads row seq_len-1 of logits computed for every position; the oracle's
    # last_token_logits must equal that row of the full final_logits, per packed sequence, and
    # the norm must be a plain RMSNorm (unit rows stay unit-RMS before the weight).
    rng = np.random.default_rng(5)
    T, H, V = 23, 64, 96
    hidden = P.round_to(rng.standard_normal((T, H)) * 3.0, "bf16")
    w = P.round_to(1.0 + 0.1 * rng.standard_normal(H), "bf16")
    lm = P.round_to(rng.standard_normal((V, H)) / 8.0, "bf16")
    cu = np.array([0, 1, 9, 10, 23])
    full = P.final_logits(hidden, w, lm, 1e-6)
    last = P.last_token_logits(hidden, cu, w, lm, 1e-6)
    assert last.shape == (4, V)
    assert np.array_equal(last, full[[0, 8, 9, 22]])
    x = hidden[22]
    ref = (x / np.sqrt(np.mean(x * x) + 1e-6) * w) @ lm.T
    assert np.allclose(last[3], ref, rtol=1e-12, atol=1e-12)
    # The candle flow (norm and logits rounded to bf16) stays within bf16 rounding of f32.
    cand = P.last_token_logits(hidden, cu, w, lm, 1e-6, flow="candle")
    assert np.abs(cand - last).max() <= 2e-2 + 1e-2 * np.abs(last).max()
