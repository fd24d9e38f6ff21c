"""CPU oracle for the projections either side of attention — TEST INFRASTRUCTURE ONLY.

A numpy restatement of CausalSelfAttention::forward up to the attention call and after it
(lltsdyp/flour src/models/common/attention.rs:75-116) and the residual add of
DecoderLayer::forward (src/models/common/transformer.rs:37-38):

* ``linear``          candle_nn::Linear: y = x W^T (+ b), W stored (out, in)   attention.rs:75-77
* ``rms_norm``        candle_nn::RmsNorm over head_dim (use_qk_norm)            attention.rs:85-92
* ``rope``            candle_nn::rotary_emb::rope (rotate-half), tables of Cache::new
                      (src/models/common/cache.rs:378-392)                      attention.rs:96-99
* ``qkv_forward``     the three above, per token, for packed tokens with their own positions
* ``o_proj_residual`` residual + o_proj(attn)                                   attention.rs:116
* ``final_logits``    CausalLM::forward's tail: final RMSNorm, lm_head, every row  model.rs:56-58
* ``last_token_logits`` the row the engine reads per sequence, as f32          engine.rs:220-222

candle-nn is not vendored (candle 0.9.2, Cargo.lock:233-236); ``rope`` restates the published
rotate-half rotation that ``rotary_emb::rope`` implements: for i < d/2,
out[i] = x[i] cos[i] - x[i + d/2] sin[i] and out[i + d/2] = x[i + d/2] cos[i] + x[i] sin[i].

``flow="f32"`` computes everything in float64 from the 16-bit inputs (the kernels compute in f32
and round once). ``flow="candle"`` rounds to the model dtype where the reference's tensors are
materialised in it: after each matmul, after the bias add, after the norm, and after each
elementwise multiply / add of the rotation (the ``half`` crate rounds every bf16 op).
Only ``tests/`` may import this module.
"""

from __future__ import annotations

import numpy as np


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to bf16 or f16 (nearest even) and return them as float64."""
    x = np.asarray(x, dtype=np.float64)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float64)
    if dtype != "bf16":
        raise ValueError(dtype)
    f = x.astype(np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    nan = np.isnan(f)
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32).astype(np.float64)
    out[nan] = np.nan
    return out


def rope_tables(head_dim: int, max_position: int, rope_theta: float, dtype: str):
    """Cache::new (cache.rs:378-392): f32 angles, cos/sin rounded to the model dtype."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    theta = (1.0 / np.power(np.float32(rope_theta), (2 * i) / np.float32(head_dim))).astype(np.float32)
    ang = (np.arange(max_position, dtype=np.float32).reshape(-1, 1) * theta.reshape(1, -1)).astype(np.float32)
    return (round_to(np.cos(ang).astype(np.float32), dtype),
            round_to(np.sin(ang).astype(np.float32), dtype))


def linear(x, w, b=None, flow="f32", dtype="bf16"):
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if flow == "candle":
        y = round_to(y, dtype)
    if b is not None:
        y = y + np.asarray(b, np.float64)
        if flow == "candle":
            y = round_to(y, dtype)
    return y


def rms_norm(x, w, eps, flow="f32", dtype="bf16"):
    """x / sqrt(mean(x^2) + eps) * w over the last axis (candle computes it in f32)."""
    x = np.asarray(x, np.float64)
    y = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(w, np.float64)
    return round_to(y, dtype) if flow == "candle" else y


def rope(x, cos, sin, flow="f32", dtype="bf16"):
    """Rotate-half RoPE of x [..., d] with per-row cos/sin [..., d/2]."""
    x = np.asarray(x, np.float64)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    if flow == "candle":
        r = lambda v: round_to(v, dtype)
        o1 = r(r(x1 * cos) - r(x2 * sin))
        o2 = r(r(x2 * cos) + r(x1 * sin))
    else:
        o1 = x1 * cos - x2 * sin
        o2 = x2 * cos + x1 * sin
    return np.concatenate([o1, o2], axis=-1)


def qkv_forward(x, weight, num_heads, num_kv_heads, head_dim, positions, cos, sin, bias=None,
                q_norm=None, k_norm=None, eps=1e-6, flow="f32", dtype="bf16"):
    """q [T, Hq, d], k [T, Hkv, d], v [T, Hkv, d] for packed tokens at their own positions.

    weight is the q_proj, k_proj, v_proj weights stacked row-wise ((Hq + 2 Hkv) d, hidden)."""
    T = x.shape[0]
    y = linear(x, weight, bias, flow, dtype)
    nq, nk = num_heads * head_dim, num_kv_heads * head_dim
    q = y[:, :nq].reshape(T, num_heads, head_dim)
    k = y[:, nq:nq + nk].reshape(T, num_kv_heads, head_dim)
    v = y[:, nq + nk:].reshape(T, num_kv_heads, head_dim)
    if q_norm is not None:
        q = rms_norm(q, q_norm, eps, flow, dtype)
    if k_norm is not None:
        k = rms_norm(k, k_norm, eps, flow, dtype)
    c = np.asarray(cos, np.float64)[positions][:, None, :]
    s = np.asarray(sin, np.float64)[positions][:, None, :]
    return rope(q, c, s, flow, dtype), rope(k, c, s, flow, dtype), v


def o_proj_residual(attn, weight, residual=None, flow="f32", dtype="bf16"):
    y = linear(attn, weight, None, flow, dtype)
    if residual is not None:
        y = y + np.asarray(residual, np.float64)
        if flow == "candle":
            y = round_to(y, dtype)
    return y


def final_logits(hidden, norm_w, lm_head, eps, flow="f32", dtype="bf16", norm_flow=None):
    """CausalLM::forward (model.rs:56-58): the final RMSNorm then lm_head, for every row.
    ``norm_flow`` overrides the flow of the norm alone (the kernels round the norm to the model
    dtype, as candle does, and keep the logits in f32)."""
    hidden = np.asarray(hidden, np.float64)
    w = np.ones(hidden.shape[-1]) if norm_w is None else norm_w
    x = rms_norm(hidden, w, eps, norm_flow or flow, dtype)
    return linear(x, lm_head, None, flow, dtype)


def last_token_logits(hidden, cu_seqlens, norm_w, lm_head, eps, flow="f32", dtype="bf16",
                      norm_flow=None):
    """engine.rs:220-222: the logits of every position, then row seq_len - 1 of each sequence
    (``logits.i((0, seq_len - 1))``), converted to f32."""
    logits = final_logits(hidden, norm_w, lm_head, eps, flow, dtype, norm_flow)
    last = np.asarray(cu_seqlens, np.int64)[1:] - 1
    return logits[last]
