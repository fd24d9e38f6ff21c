"""Shared helpers for the GPU parity tests: run the oracle on the same inputs as the kernels."""

import numpy as np
import torch

import oracle
from flour_b200.workloads import ORACLE_DT, to_numpy


def oracle_attention(q, k_cache, v_cache, cu_seqlens, context_lens, block_tables, n_rep, scale,
                     score_mode=0):
    """Run oracle.paged_attention on device tensors; returns float32 numpy output."""
    dt = ORACLE_DT[q.dtype]
    out, err = oracle.paged_attention(
        to_numpy(q), to_numpy(k_cache), to_numpy(v_cache), to_numpy(cu_seqlens),
        to_numpy(context_lens), to_numpy(block_tables), n_rep, scale, dtype=dt,
        score_mode=score_mode)
    assert err == 0, err
    return oracle.to_f32(out, dt)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def max_abs(a, b) -> float:
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())
