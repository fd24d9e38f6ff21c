"""torch-facing wrappers over the C ABI (device memory and streams come from torch).

Every function here calls exactly one ``fa_*`` entry point of libflour_attn.so on the current
torch CUDA stream; there is no Python compute path.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import FaKvLayer, check, lib

_DTYPES = {torch.float32: _lib.FA_F32, torch.bfloat16: _lib.FA_BF16, torch.float16: _lib.FA_F16}


def fa_dtype(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"unsupported dtype {dtype}") from None


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def layer_desc(k_cache: torch.Tensor, v_cache: torch.Tensor) -> FaKvLayer:
    """``fa_kv_layer`` for one layer's slabs of shape [num_blocks, kv_heads, bs, head_dim]."""
    if k_cache.shape != v_cache.shape or k_cache.dtype != v_cache.dtype:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "k_cache and v_cache differ in shape or dtype")
    if k_cache.dim() != 4 or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise _lib.FlourAttnError(_lib.FA_EINVAL,
                                  "cache slabs must be contiguous [num_blocks, kv_heads, bs, d]")
    nb, kvh, bs, d = k_cache.shape
    return FaKvLayer(k_cache.data_ptr(), v_cache.data_ptr(), nb, kvh, bs, d, fa_dtype(k_cache.dtype))


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"{name} must be a contiguous int32 tensor")
    return t


# ---- block writes / copies ----------------------------------------------------------------

def reshape_and_cache(k_cache, v_cache, key, value, slot_mapping, stream=None) -> None:
    """Scatter key/value rows [T, kv_heads, d] (any token/head strides, unit stride on d) into
    their pool slots; slot -1 skips a token. PagedKvPool::write, paged.rs:186-204."""
    layer = layer_desc(k_cache, v_cache)
    if key.stride(-1) != 1 or value.stride(-1) != 1:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "key/value need unit stride on head_dim")
    if key.dtype != k_cache.dtype or value.dtype != k_cache.dtype:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "key/value dtype differs from the pool dtype")
    sm = _i32(slot_mapping, "slot_mapping")
    check(lib().fa_reshape_and_cache(ctypes.byref(layer), _ptr(key), _ptr(value), key.stride(0),
                                     key.stride(1), value.stride(0), value.stride(1), _ptr(sm),
                                     sm.numel(), _stream(stream)), "reshape_and_cache")


def copy_blocks(k_caches, v_caches, block_mapping, stream=None) -> None:
    """Copy whole blocks (src, dst) = block_mapping[i] in every layer, K and V."""
    layers = (FaKvLayer * len(k_caches))(*[layer_desc(k, v) for k, v in zip(k_caches, v_caches)])
    bm = _i32(block_mapping, "block_mapping")
    check(lib().fa_copy_blocks(layers, len(k_caches), _ptr(bm), bm.numel() // 2, _stream(stream)),
          "copy_blocks")


def write_block(k_cache, v_cache, block_id: int, key, value, stream=None) -> None:
    """PagedKvPool::write_block: key/value (kv_heads, bs, d), host (pinned or not) or device."""
    layer = layer_desc(k_cache, v_cache)
    check(lib().fa_write_block(ctypes.byref(layer), block_id, _ptr(key.contiguous()),
                               _ptr(value.contiguous()), _stream(stream)), "write_block")


def read_block(k_cache, v_cache, block_id: int, key_out, value_out, stream=None) -> None:
    layer = layer_desc(k_cache, v_cache)
    check(lib().fa_read_block(ctypes.byref(layer), block_id, _ptr(key_out), _ptr(value_out),
                              _stream(stream)), "read_block")


def bundle_payload_bytes(k_caches, v_caches, num_blocks: int) -> int:
    layer = layer_desc(k_caches[0], v_caches[0])
    return int(lib().fa_bundle_payload_bytes(ctypes.byref(layer), len(k_caches), num_blocks))


def export_bundle_payload(k_caches, v_caches, block_ids, payload=None, stream=None):
    """FLKV payload of the physical blocks `block_ids` (logical order) of every layer, in one
    launch: for block, for layer, K then V (kv_heads, bs, d). Returns the device uint8 payload
    (`payload` if given); the caller copies it to the host in one transfer."""
    layers = (FaKvLayer * len(k_caches))(*[layer_desc(k, v) for k, v in zip(k_caches, v_caches)])
    ids = _i32(block_ids, "block_ids")
    n = bundle_payload_bytes(k_caches, v_caches, ids.numel())
    if payload is None:
        payload = torch.empty(n, dtype=torch.uint8, device=k_caches[0].device)
    elif payload.numel() * payload.element_size() < n or not payload.is_contiguous():
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"payload must be contiguous with >= {n} bytes")
    check(lib().fa_export_bundle_payload(layers, len(k_caches), _ptr(ids), ids.numel(),
                                         _ptr(payload), _stream(stream)), "export_bundle_payload")
    return payload


def import_bundle_payload(k_caches, v_caches, block_ids, payload, stream=None) -> None:
    """The mirror of export_bundle_payload: payload (device) -> physical blocks `block_ids` of
    every layer, in one launch."""
    layers = (FaKvLayer * len(k_caches))(*[layer_desc(k, v) for k, v in zip(k_caches, v_caches)])
    ids = _i32(block_ids, "block_ids")
    n = bundle_payload_bytes(k_caches, v_caches, ids.numel())
    if payload.numel() * payload.element_size() < n or not payload.is_contiguous():
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"payload must be contiguous with >= {n} bytes")
    check(lib().fa_import_bundle_payload(layers, len(k_caches), _ptr(ids), ids.numel(),
                                         _ptr(payload), _stream(stream)), "import_bundle_payload")


# ---- attention ----------------------------------------------------------------------------

def workspace_size(num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                   max_context_len: int, max_seqlen_q: int) -> int:
    return int(lib().fa_paged_attention_workspace_size(num_seqs, num_heads, num_kv_heads,
                                                       head_dim, max_context_len, max_seqlen_q))


class Workspace:
    """Caller-owned, zero-initialised scratch for the split-K partials (grown on demand).
    One Workspace per stream: concurrent calls must not share it."""

    def __init__(self, device=None):
        self.device = torch.device(device if device is not None else "cuda")
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int) -> torch.Tensor | None:
        if nbytes == 0:
            return self.buf
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            # A fresh zero-filled buffer: bookkeeping kept for an earlier buffer at the same
            # address (the caching allocator reuses addresses) no longer applies.
            check(lib().fa_workspace_reset(_ptr(self.buf)), "workspace_reset")
        return self.buf


def _ws_args(ws: Workspace | None, need: int):
    if need == 0:
        return None, 0
    if ws is None:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"a workspace of {need} bytes is required")
    buf = ws.get(need)
    return _ptr(buf), buf.numel()


def paged_decode(query, k_cache, v_cache, block_tables, context_lens, n_rep: int, scale: float,
                 max_context_len: int, workspace: Workspace | None = None, out=None,
                 stream=None, score_flow: int = _lib.FA_SCORES_F32):
    """One query token per sequence: query [B, Hq, d] -> out [B, Hq, d]. `score_flow`:
    FA_SCORES_F32 (default) or FA_SCORES_REFERENCE (the reference's bf16/f16 score rounding,
    src/backend/cpu.rs:84-85)."""
    layer = layer_desc(k_cache, v_cache)
    query = query.contiguous()
    out = torch.empty_like(query) if out is None else out
    bt, cl = _i32(block_tables, "block_tables"), _i32(context_lens, "context_lens")
    B, hq, d = query.shape
    need = workspace_size(B, hq, k_cache.shape[1], d, max_context_len, 1)
    wp, wn = _ws_args(workspace, need)
    check(lib().fa_paged_decode(ctypes.byref(layer), _ptr(query), _ptr(out), _ptr(cl), _ptr(bt),
                                bt.shape[1], B, hq, n_rep, max_context_len, scale, score_flow,
                                wp, wn, _stream(stream)), "paged_decode")
    return out


def paged_decode_append(query, k_cache, v_cache, key, value, block_tables, context_lens,
                        n_rep: int, scale: float, max_context_len: int,
                        workspace: Workspace | None = None, out=None, stream=None,
                        score_flow: int = _lib.FA_SCORES_F32):
    """Write each sequence's new token (key/value [B, kv_heads, d], any token/head strides,
    unit stride on d) at position context_lens[b]-1, then decode query [B, Hq, d] over the whole
    context, in one launch: reshape_and_cache + paged_decode of a decode step."""
    layer = layer_desc(k_cache, v_cache)
    query = query.contiguous()
    if key.stride(-1) != 1 or value.stride(-1) != 1:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "key/value need unit stride on head_dim")
    if key.dtype != k_cache.dtype or value.dtype != k_cache.dtype:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "key/value dtype differs from the pool dtype")
    out = torch.empty_like(query) if out is None else out
    bt, cl = _i32(block_tables, "block_tables"), _i32(context_lens, "context_lens")
    B, hq, d = query.shape
    need = workspace_size(B, hq, k_cache.shape[1], d, max_context_len, 1)
    wp, wn = _ws_args(workspace, need)
    check(lib().fa_paged_decode_append(ctypes.byref(layer), _ptr(query), _ptr(key), _ptr(value),
                                       key.stride(0), key.stride(1), value.stride(0),
                                       value.stride(1), _ptr(out), _ptr(cl), _ptr(bt),
                                       bt.shape[1], B, hq, n_rep, max_context_len, scale,
                                       score_flow, wp, wn, _stream(stream)),
          "paged_decode_append")
    return out


def paged_decode_noalloc(query, k_cache, v_cache, block_tables, context_lens, n_rep: int,
                        scale: float, max_context_len: int, out=None, stream=None):
    """paged_decode without a workspace: the split-K scratch is the library's fixed buffer
    (fa_paged_decode_noalloc). Calls on different streams must not overlap on the GPU."""
    layer = layer_desc(k_cache, v_cache)
    query = query.contiguous()
    out = torch.empty_like(query) if out is None else out
    bt, cl = _i32(block_tables, "block_tables"), _i32(context_lens, "context_lens")
    B, hq, d = query.shape
    check(lib().fa_paged_decode_noalloc(ctypes.byref(layer), _ptr(query), _ptr(out), _ptr(cl),
                                        _ptr(bt), bt.shape[1], B, hq, n_rep, max_context_len,
                                        scale, _stream(stream)), "paged_decode_noalloc")
    return out


def paged_prefill(query, k_cache, v_cache, cu_seqlens_q, context_lens, block_tables, n_rep: int,
                  scale: float, max_seqlen_q: int, max_context_len: int,
                  workspace: Workspace | None = None, out=None, stream=None,
                  score_flow: int = _lib.FA_SCORES_F32):
    """Varlen causal attention of packed suffix queries [Tq, Hq, d] over prefix+suffix KV."""
    layer = layer_desc(k_cache, v_cache)
    query = query.contiguous()
    out = torch.empty_like(query) if out is None else out
    cu = _i32(cu_seqlens_q, "cu_seqlens_q")
    bt, cl = _i32(block_tables, "block_tables"), _i32(context_lens, "context_lens")
    tq, hq, d = query.shape
    S = cl.numel()
    need = workspace_size(S, hq, k_cache.shape[1], d, max_context_len, max_seqlen_q)
    wp, wn = _ws_args(workspace, need)
    check(lib().fa_paged_prefill(ctypes.byref(layer), _ptr(query), _ptr(out), _ptr(cu), _ptr(cl),
                                 _ptr(bt), bt.shape[1], S, hq, n_rep, tq, max_seqlen_q,
                                 max_context_len, scale, score_flow, wp, wn, _stream(stream)),
          "paged_prefill")
    return out


def paged_attention_varlen(query, k_cache, v_cache, cu_seqlens_q, context_lens, block_tables,
                           n_rep: int, scale: float, max_seqlen_q: int, max_context_len: int,
                           workspace: Workspace | None = None, out=None, stream=None,
                           score_flow: int = _lib.FA_SCORES_F32):
    """The general entry (fa_paged_attention): decode or prefill chosen by the library."""
    layer = layer_desc(k_cache, v_cache)
    query = query.contiguous()
    out = torch.empty_like(query) if out is None else out
    cu = _i32(cu_seqlens_q, "cu_seqlens_q")
    bt, cl = _i32(block_tables, "block_tables"), _i32(context_lens, "context_lens")
    tq, hq, d = query.shape
    S = cl.numel()
    need = workspace_size(S, hq, k_cache.shape[1], d, max_context_len,
                          1 if (max_seqlen_q == 1 and tq == S) else max_seqlen_q)
    wp, wn = _ws_args(workspace, need)
    check(lib().fa_paged_attention(ctypes.byref(layer), _ptr(query), _ptr(out), _ptr(cu), _ptr(cl),
                                   _ptr(bt), bt.shape[1], S, hq, n_rep, tq, max_seqlen_q,
                                   max_context_len, scale, score_flow, wp, wn, _stream(stream)),
          "paged_attention")
    return out


def device_status(clear: bool = True, stream=None) -> int:
    """FA_DEVERR_* bits the kernels reported on the current device (waits for the stream)."""
    v = ctypes.c_int32(0)
    st = lib().fa_device_status(ctypes.byref(v), 1 if clear else 0, _stream(stream))
    if st not in (_lib.FA_OK, _lib.FA_EDEVICE, _lib.FA_ETIMEOUT):
        check(st, "device_status")
    return int(v.value)


def default_scale(head_dim: int) -> float:
    """1/sqrt(head_dim), the scale attention.rs:108 passes."""
    return 1.0 / math.sqrt(head_dim)


# ---- the projections either side of attention (CausalSelfAttention::forward) --------------

def _c16(t: torch.Tensor | None, name: str, dtype: torch.dtype) -> torch.Tensor | None:
    if t is None:
        return None
    if t.dtype != dtype or not t.is_contiguous() or not t.is_cuda:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"{name} must be a contiguous CUDA {dtype} tensor")
    return t


def qkv_rope_cache(x, weight, k_cache, v_cache, positions, slot_mapping, num_heads: int,
                   rope_cos, rope_sin, bias=None, q_norm_weight=None, k_norm_weight=None,
                   rms_eps: float = 1e-6, q_out=None, stream=None) -> torch.Tensor:
    """Fused q/k/v projection + (optional) per-head RMSNorm + RoPE + reshape_and_cache.

    x [T, hidden]; weight [(num_heads + 2*kv_heads) * d, hidden] (q_proj, k_proj, v_proj rows
    stacked); positions / slot_mapping int32 [T]; rope_cos / rope_sin f32 [max_position, d/2].
    Returns q [T, num_heads, d]; K/V land in the pool. attention.rs:75-104."""
    layer = layer_desc(k_cache, v_cache)
    dt = k_cache.dtype
    x = _c16(x, "x", dt)
    weight = _c16(weight, "weight", dt)
    for name, t in (("bias", bias), ("q_norm_weight", q_norm_weight), ("k_norm_weight", k_norm_weight)):
        _c16(t, name, dt)
    if rope_cos.dtype != torch.float32 or rope_sin.dtype != torch.float32 or \
            not (rope_cos.is_contiguous() and rope_sin.is_contiguous()) or rope_cos.shape != rope_sin.shape:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "rope tables must be contiguous f32 [max_pos, d/2]")
    T, hidden = x.shape
    d = k_cache.shape[-1]
    n_out = (num_heads + 2 * k_cache.shape[1]) * d
    if tuple(weight.shape) != (n_out, hidden) or (bias is not None and tuple(bias.shape) != (n_out,)):
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"weight must be [{n_out}, {hidden}] (bias [{n_out}])")
    for name, t in (("q_norm_weight", q_norm_weight), ("k_norm_weight", k_norm_weight)):
        if t is not None and tuple(t.shape) != (d,):
            raise _lib.FlourAttnError(_lib.FA_EINVAL, f"{name} must be [{d}]")
    if rope_cos.dim() != 2 or rope_cos.shape[1] != d // 2:
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"rope tables must be [max_pos, {d // 2}]")
    if q_out is None:
        q_out = torch.empty((T, num_heads, d), dtype=dt, device=x.device)
    w = _lib.FaQkvWeights(weight.data_ptr(), bias.data_ptr() if bias is not None else None,
                          q_norm_weight.data_ptr() if q_norm_weight is not None else None,
                          k_norm_weight.data_ptr() if k_norm_weight is not None else None,
                          float(rms_eps), hidden, num_heads, rope_cos.data_ptr(),
                          rope_sin.data_ptr(), rope_cos.shape[0])
    check(lib().fa_qkv_rope_cache(ctypes.byref(layer), ctypes.byref(w), _ptr(x),
                                  _ptr(_i32(positions, "positions")),
                                  _ptr(_i32(slot_mapping, "slot_mapping")), T, _ptr(q_out),
                                  _stream(stream)),
          "qkv_rope_cache")
    return q_out


def last_token_logits(hidden, cu_seqlens, lm_head, norm_weight=None, rms_eps: float = 1e-6,
                      normed_out=None, logits_out=None, stream=None) -> torch.Tensor:
    """f32 logits [S, vocab] of each sequence's last token: final RMSNorm + lm_head
    (model.rs:56-58) on the rows the engine reads (engine.rs:220-222). hidden [T, H] packed,
    cu_seqlens int32 [S + 1], lm_head [vocab, H]."""
    dt = hidden.dtype
    hidden = _c16(hidden, "hidden", dt)
    lm_head = _c16(lm_head, "lm_head", dt)
    _c16(norm_weight, "norm_weight", dt)
    cu = _i32(cu_seqlens, "cu_seqlens")
    T, H = hidden.shape
    S = cu.numel() - 1
    V = lm_head.shape[0]
    if lm_head.shape[1] != H or (norm_weight is not None and tuple(norm_weight.shape) != (H,)):
        raise _lib.FlourAttnError(_lib.FA_EINVAL, f"lm_head must be [vocab, {H}] (norm_weight [{H}])")
    if normed_out is None:
        normed_out = torch.empty((S, H), dtype=dt, device=hidden.device)
    if logits_out is None:
        logits_out = torch.empty((S, V), dtype=torch.float32, device=hidden.device)
    check(lib().fa_last_token_logits(_ptr(hidden), _ptr(cu), S, T, _ptr(norm_weight),
                                     float(rms_eps), _ptr(lm_head), H, V, fa_dtype(dt),
                                     _ptr(normed_out), _ptr(logits_out), _stream(stream)),
          "last_token_logits")
    return logits_out


def o_proj_residual(attn, weight, residual=None, out=None, stream=None) -> torch.Tensor:
    """out = residual + attn @ weight^T (residual optional, may alias out).

    attn [T, in_features] (heads concatenated), weight [out_features, in_features].
    attention.rs:116 + transformer.rs:37-38."""
    dt = attn.dtype
    attn = _c16(attn, "attn", dt)
    weight = _c16(weight, "weight", dt)
    _c16(residual, "residual", dt)
    T, fin = attn.shape
    fout = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != fin or \
            (residual is not None and tuple(residual.shape) != (T, fout)):
        raise _lib.FlourAttnError(_lib.FA_EINVAL, "weight must be [out, in], residual [T, out]")
    if out is None:
        out = torch.empty((T, fout), dtype=dt, device=attn.device)
    check(lib().fa_o_proj_residual(_ptr(attn), _ptr(weight), _ptr(residual), _ptr(out), T, fin,
                                   fout, fa_dtype(dt), _stream(stream)),
          "o_proj_residual")
    return out
