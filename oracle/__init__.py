"""CPU oracle for the paged KV pool + paged attention path — TEST INFRASTRUCTURE ONLY.

ctypes bindings over ``oracle/liboracle.so`` (built from ``ref_paged_attention.cpp`` and
``flkv_bundle.cpp`` by ``oracle/Makefile``), a C++ restatement of the reference:

* ``paged_attention``      lltsdyp/flour src/backend/cpu.rs:57-112
* ``causal_attention``     src/backend/cpu.rs:24-42
* ``slot`` / ``slots``     src/models/common/paged.rs:114-121
* ``pool_write_literal``   src/models/common/paged.rs:186-204 (as written, reference layout)
* ``reshape_and_cache``    per-slot scatter on the build layout
* ``copy_blocks``          paged.rs:211-240 + 266-279
* ``bundle_export/import`` src/kv_cache/bundle.rs:15-22, src/models/common/cache.rs:166-349

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this
package; the CUDA product never does. Arrays are numpy; bf16 and f16 are carried as uint16.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

DT_F32, DT_BF16, DT_F16 = 0, 1, 2
ERR_BLOCK_ID, ERR_CONTEXT, ERR_SLOT, ERR_SEQLEN, ERR_PAIR = 0x1, 0x2, 0x4, 0x10, 0x20

_lib = None

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        L = _lib
        L.oracle_slot.restype = _I64
        L.oracle_slot.argtypes = [_P, _I32, _I64]
        L.oracle_slots.restype = None
        L.oracle_slots.argtypes = [_P, _I32, _I64, _I64, _P]
        L.oracle_pool_write_literal.restype = _I32
        L.oracle_pool_write_literal.argtypes = [_P, _P, _I32, _I64, _I32, _I32, _P, _I64, _P, _P]
        L.oracle_reshape_and_cache.restype = _I32
        L.oracle_reshape_and_cache.argtypes = [_P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P,
                                               _I64, _I64, _I64, _I64, _P, _I64]
        L.oracle_copy_blocks.restype = _I32
        L.oracle_copy_blocks.argtypes = [_P, _P, _I32, _I32, _I64, _P, _I32]
        L.oracle_causal_attention.restype = _I32
        L.oracle_causal_attention.argtypes = [_I32, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                              ctypes.c_float, _P]
        L.oracle_paged_attention.restype = _I32
        L.oracle_paged_attention.argtypes = [_I32, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                             _I32, _I32, _P, _P, _P, _I32, _I32, ctypes.c_float,
                                             _I32]
        L.oracle_bundle_export.restype = _I64
        L.oracle_bundle_export.argtypes = [_P, _P, _I32, _I64, _P, _I32, _P]
        L.oracle_bundle_import.restype = None
        L.oracle_bundle_import.argtypes = [_P, _P, _I32, _I64, _P, _I32, _P]
        L.oracle_max_threads.restype = _I32
    return _lib


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _dt_of(a: np.ndarray, dtype: int | None) -> int:
    if dtype is not None:
        return dtype
    if a.dtype == np.float32:
        return DT_F32
    raise ValueError("uint16 arrays need an explicit dtype (DT_BF16 or DT_F16)")


# ---- dtype helpers (numpy, round-to-nearest-even like half::bf16::from_f32) ---------------

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def to_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == DT_F32:
        return np.asarray(a, dtype=np.float32)
    return bf16_to_f32(a) if dtype == DT_BF16 else f16_to_f32(a)


def from_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == DT_F32:
        return np.ascontiguousarray(a, dtype=np.float32)
    return f32_to_bf16(a) if dtype == DT_BF16 else f32_to_f16(a)


# ---- block table (paged.rs:114-121) -----------------------------------------------------

def slot(blocks, block_size: int, pos: int) -> int:
    b = np.ascontiguousarray(blocks, dtype=np.int32)
    return int(lib().oracle_slot(_ptr(b), block_size, pos))


def slots(blocks, block_size: int, start: int, end: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.int32)
    out = np.zeros(max(end - start, 0), dtype=np.uint32)
    lib().oracle_slots(_ptr(b), block_size, start, end, _ptr(out))
    return out


# ---- pool writes ------------------------------------------------------------------------

def pool_write_literal(k_pool: np.ndarray, v_pool: np.ndarray, slot_list, k: np.ndarray,
                       v: np.ndarray) -> int:
    """PagedKvPool::write exactly as written (paged.rs:186-204), reference layout.

    k_pool/v_pool: (kv_heads, num_slots, d); k/v: (kv_heads, n, d). In place."""
    kv_heads, num_slots, d = k_pool.shape
    s = np.ascontiguousarray(slot_list, dtype=np.uint32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    return int(lib().oracle_pool_write_literal(_ptr(k_pool), _ptr(v_pool), kv_heads, num_slots, d,
                                               k_pool.itemsize, _ptr(s), len(s), _ptr(k), _ptr(v)))


def reshape_and_cache(k_cache: np.ndarray, v_cache: np.ndarray, key: np.ndarray,
                      value: np.ndarray, slot_mapping) -> int:
    """Per-slot scatter into the build layout [num_blocks, kv_heads, bs, d]. key/value are
    [T, kv_heads, d] contiguous. In place; returns ERR_* bits."""
    nb, kvh, bs, d = k_cache.shape
    key = np.ascontiguousarray(key)
    value = np.ascontiguousarray(value)
    sm = np.ascontiguousarray(slot_mapping, dtype=np.int32)
    return int(lib().oracle_reshape_and_cache(_ptr(k_cache), _ptr(v_cache), nb, kvh, bs, d,
                                              k_cache.itemsize, _ptr(key), _ptr(value),
                                              kvh * d, d, kvh * d, d, _ptr(sm), len(sm)))


def copy_blocks(k_caches: list, v_caches: list, pairs) -> int:
    p = np.ascontiguousarray(pairs, dtype=np.int32).reshape(-1, 2)
    nb = k_caches[0].shape[0]
    block_bytes = k_caches[0][0].nbytes
    kp = (ctypes.c_void_p * len(k_caches))(*[a.ctypes.data for a in k_caches])
    vp = (ctypes.c_void_p * len(v_caches))(*[a.ctypes.data for a in v_caches])
    return int(lib().oracle_copy_blocks(kp, vp, len(k_caches), nb, block_bytes, _ptr(p), len(p)))


# ---- attention ----------------------------------------------------------------------------

def causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask, scale: float,
                     n_rep: int = 1, dtype: int | None = None) -> np.ndarray:
    """cpu.rs:24-42 for one batch element: q (H, sq, d), k/v (H/n_rep, kv, d)."""
    dt = _dt_of(q, dtype)
    q = np.ascontiguousarray(q)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    h, sq, d = q.shape
    kv = k.shape[1]
    out = np.zeros_like(q)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    rc = lib().oracle_causal_attention(dt, _ptr(q), _ptr(k), _ptr(v), _ptr(out), h, n_rep, sq, kv,
                                       d, scale, _ptr(m))
    if rc != 0:
        raise ValueError(f"oracle_causal_attention rejected arguments ({rc})")
    return out


def paged_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, cu_seqlens_q,
                    context_lens, block_tables, n_rep: int, scale: float,
                    dtype: int | None = None, score_mode: int = 0, threads: int = 0):
    """cpu.rs:57-112 over a varlen batch. q: [total_q, Hq, d]; caches
    [num_blocks, Hkv, bs, d]. Returns (out, err_bits)."""
    dt = _dt_of(q, dtype)
    q = np.ascontiguousarray(q)
    nb, kvh, bs, d = k_cache.shape
    hq = q.shape[1]
    cu = np.ascontiguousarray(cu_seqlens_q, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    if bt.ndim == 1:
        bt = bt.reshape(len(cl), -1)
    out = np.zeros_like(q)
    rc = lib().oracle_paged_attention(dt, score_mode, _ptr(q), _ptr(out), _ptr(k_cache),
                                      _ptr(v_cache), nb, kvh, bs, d, hq, n_rep, _ptr(cu), _ptr(cl),
                                      _ptr(bt), bt.shape[1], len(cl), scale, threads)
    if rc < 0:
        raise ValueError("oracle_paged_attention rejected arguments")
    return out, rc


# ---- FLKV bundle payload ------------------------------------------------------------------

def bundle_export(k_caches: list, v_caches: list, block_ids) -> np.ndarray:
    ids = np.ascontiguousarray(block_ids, dtype=np.int32)
    block_bytes = k_caches[0][0].nbytes
    out = np.zeros(len(ids) * len(k_caches) * 2 * block_bytes, dtype=np.uint8)
    kp = (ctypes.c_void_p * len(k_caches))(*[a.ctypes.data for a in k_caches])
    vp = (ctypes.c_void_p * len(v_caches))(*[a.ctypes.data for a in v_caches])
    n = lib().oracle_bundle_export(kp, vp, len(k_caches), block_bytes, _ptr(ids), len(ids),
                                   _ptr(out))
    assert n == out.nbytes
    return out


def bundle_import(k_caches: list, v_caches: list, block_ids, payload: np.ndarray) -> None:
    ids = np.ascontiguousarray(block_ids, dtype=np.int32)
    block_bytes = k_caches[0][0].nbytes
    kp = (ctypes.c_void_p * len(k_caches))(*[a.ctypes.data for a in k_caches])
    vp = (ctypes.c_void_p * len(v_caches))(*[a.ctypes.data for a in v_caches])
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    lib().oracle_bundle_import(kp, vp, len(k_caches), block_bytes, _ptr(ids), len(ids),
                               _ptr(payload))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def cpu_threads() -> int:
    """Host threads the oracle may use (respects OMP_NUM_THREADS / affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
