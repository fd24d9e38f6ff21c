"""ctypes binding of libflour_attn.so (the C ABI declared in include/flour_attn.h).

Loading fails loudly when the library has not been built: there is no Python or CPU fallback
for any entry point.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libflour_attn.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "flour_attn.h"

FA_OK, FA_EINVAL, FA_ERANGE, FA_ECUDA, FA_ETIMEOUT, FA_EUNSUPPORTED, FA_EDEVICE = 0, -1, -2, -3, -4, -5, -6
FA_F32, FA_BF16, FA_F16 = 0, 1, 2
FA_SCORES_F32, FA_SCORES_REFERENCE = 0, 1
FA_DEVERR_BLOCK_ID = 0x1
FA_DEVERR_CONTEXT = 0x2
FA_DEVERR_SLOT = 0x4
FA_DEVERR_TIMEOUT = 0x8
FA_DEVERR_SEQLEN = 0x10
FA_DEVERR_PAIR = 0x20
FA_DEVERR_POSITION = 0x40
FA_DEVERR_LAUNCH = 0x80
FA_MAX_COPY_LAYERS = 128
FA_NOALLOC_DECODE_SCRATCH_BYTES = 8 * 1024 * 1024

# Every function the header declares, with its ctypes signature.
_P, _I32, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float


class FaKvLayer(ctypes.Structure):
    """``fa_kv_layer``: one layer of the pool, K/V slabs [num_blocks, kv_heads, bs, head_dim]."""

    _fields_ = [
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


_LP = ctypes.POINTER(FaKvLayer)


class FaQkvWeights(ctypes.Structure):
    """``fa_qkv_weights``: one layer's stacked q/k/v projection weights and RoPE tables."""

    _fields_ = [
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("q_norm_weight", ctypes.c_void_p),
        ("k_norm_weight", ctypes.c_void_p),
        ("rms_eps", ctypes.c_float),
        ("hidden", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("max_position", ctypes.c_int32),
    ]


_WP = ctypes.POINTER(FaQkvWeights)

FA_MAX_TP = 8
FA_TP_PUBLISH, FA_TP_WAIT = 1, 2


class FaIpcHandle(ctypes.Structure):
    """``fa_ipc_handle``: a CUDA IPC memory handle, 64 opaque bytes."""

    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class FaTpGroup(ctypes.Structure):
    """``fa_tp_group``: the ranks' output buffers and flag arrays as mapped in this process."""

    _fields_ = [
        ("tp", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("out", ctypes.c_void_p * FA_MAX_TP),
        ("flags", ctypes.c_void_p * FA_MAX_TP),
        ("epoch_counter", ctypes.c_void_p),
    ]


_HP = ctypes.POINTER(FaIpcHandle)
_GP = ctypes.POINTER(FaTpGroup)

SIGNATURES = {
    "fa_abi_version": (_I32, []),
    "fa_status_string": (ctypes.c_char_p, [_I32]),
    "fa_last_error_message": (ctypes.c_char_p, []),
    "fa_device_status": (_I32, [ctypes.POINTER(_I32), _I32, _P]),
    "fa_reshape_and_cache": (_I32, [_LP, _P, _P, _I64, _I64, _I64, _I64, _P, _I32, _P]),
    "fa_copy_blocks": (_I32, [_LP, _I32, _P, _I32, _P]),
    "fa_write_block": (_I32, [_LP, _I32, _P, _P, _P]),
    "fa_read_block": (_I32, [_LP, _I32, _P, _P, _P]),
    "fa_paged_attention_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32, _I32]),
    "fa_paged_attention": (_I32, [_LP, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                  _I32, _F, _I32, _P, _SZ, _P]),
    "fa_paged_decode": (_I32, [_LP, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P,
                               _SZ, _P]),
    "fa_paged_decode_append": (_I32, [_LP, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I32,
                                      _I32, _I32, _I32, _I32, _F, _I32, _P, _SZ, _P]),
    "fa_paged_decode_noalloc": (_I32, [_LP, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _P]),
    "fa_paged_prefill": (_I32, [_LP, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                                _F, _I32, _P, _SZ, _P]),
    "fa_bundle_payload_bytes": (_SZ, [_LP, _I32, _I32]),
    "fa_export_bundle_payload": (_I32, [_LP, _I32, _P, _I32, _P, _P]),
    "fa_import_bundle_payload": (_I32, [_LP, _I32, _P, _I32, _P, _P]),
    "fa_gemm_tile_width": (_I32, [_I32, _I32, _I32]),
    "fa_workspace_reset": (_I32, [_P]),
    "fa_qkv_rope_cache": (_I32, [_LP, _WP, _P, _P, _P, _I32, _P, _P]),
    "fa_o_proj_residual": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _P]),
    "fa_last_token_logits": (_I32, [_P, _P, _I32, _I32, _P, _F, _P, _I32, _I32, _I32, _P, _P, _P]),
    "fa_ipc_alloc": (_I32, [_SZ, ctypes.POINTER(_P), _HP]),
    "fa_ipc_free": (_I32, [_P]),
    "fa_ipc_open": (_I32, [_HP, ctypes.POINTER(_P)]),
    "fa_ipc_close": (_I32, [_P]),
    "fa_paged_decode_tp": (_I32, [_GP, _LP, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32,
                                  _P, _SZ, _P]),
    "fa_tp_sync": (_I32, [_GP, ctypes.c_uint32, _I32, _I64, _P]),
}


class FlourAttnError(RuntimeError):
    """A non-OK ``fa_status``; ``.status`` holds the code, the message the library's text."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m flour_b200.build` "
                "(there is no fallback implementation)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != FA_OK:
        L = lib()
        detail = L.fa_last_error_message().decode() or L.fa_status_string(status).decode()
        raise FlourAttnError(status, f"{what}: {detail} (status {status})")
