"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

1. ``reference_literals.json`` — the known-answer values the reference's own unit tests assert
   (lltsdyp/flour has no golden-vector files; these literals are its pins):
   * causal attention known answer          src/backend/cpu.rs:245-261
   * slot-mapping golden values              src/models/common/paged.rs:378-394
   * write-then-gather exact values          src/models/common/paged.rs:287-306
   * write_block / block_view exact values   src/models/common/paged.rs:309-331
   * bundle export values (layer*1000 + i)   src/models/common/cache.rs:727-783
2. ``dense_f64_cases.npz`` — seeded small attention problems with outputs from an independent
   float64 numpy restatement of the reference's dense causal SDPA (cpu.rs:24-42 plus the mask
   rule of cpu.rs:149-165). The reference's own tests require paged == dense within 1e-4
   (cpu.rs:183-188); the oracle's paged fold is pinned to these fixtures at that tolerance.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def dense_f64(q, k, v, n_rep, scale):
    """q (H, sq, d), k/v (H/n_rep, kv, d) -> (H, sq, d), float64, causal with offset."""
    h, sq, d = q.shape
    kv = k.shape[1]
    off = kv - sq
    out = np.zeros((h, sq, d))
    for hh in range(h):
        kh = hh // n_rep
        s = (q[hh].astype(np.float64) @ k[kh].astype(np.float64).T) * scale
        mask = np.arange(kv)[None, :] > (np.arange(sq)[:, None] + off)
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[hh] = p @ v[kh].astype(np.float64)
    return out


def literals() -> dict:
    return {
        "causal_known_answer": {
            "source": "src/backend/cpu.rs:245-261",
            "q": [1.0, 1.0], "k": [1.0, 1.0], "v": [10.0, 20.0],
            "mask": [[0, 1], [0, 0]], "scale": 1.0, "expected": [10.0, 15.0], "tol": 1e-4,
        },
        "slot_mapping": {
            "source": "src/models/common/paged.rs:378-394",
            "blocks": [5, 3], "block_size": 2,
            "slot": {"0": 10, "1": 11, "2": 6, "3": 7}, "slots_0_3": [10, 11, 6],
        },
        "write_then_gather": {
            "source": "src/models/common/paged.rs:287-306",
            "num_slots": 4, "kv_heads": 1, "head_dim": 2,
            "k": [1.0, 2.0, 3.0, 4.0], "v": [5.0, 6.0, 7.0, 8.0], "slots": [2, 0],
            "gather_slots": [0, 2], "gk": [3.0, 4.0, 1.0, 2.0], "gv": [7.0, 8.0, 5.0, 6.0],
        },
        "write_block_round_trip": {
            "source": "src/models/common/paged.rs:309-331",
            "num_slots": 4, "kv_heads": 1, "head_dim": 2, "block_size": 2, "block_id": 1,
            "k": [1.0, 2.0, 3.0, 4.0], "v": [5.0, 6.0, 7.0, 8.0],
            "untouched_block": 0, "untouched_value": 0.0,
        },
        "bundle_export_values": {
            "source": "src/models/common/cache.rs:727-783",
            "kv_heads": 2, "head_dim": 4, "num_layers": 2, "tokens": 32, "block_size": 16,
            "k_formula": "layer*1000 + i over (1, kv_heads, 32, head_dim) row-major",
            "v_offset": 0.25,
        },
    }


def dense_cases(rng: np.random.Generator) -> dict:
    """Shapes: the reference's own tests (cpu.rs:190-242) and C1-like GQA cases."""
    cases = {}
    specs = [
        # name, H, Hkv, sq, kv, d, bs
        ("ref_prefill", 2, 2, 5, 5, 4, 2),      # cpu.rs:190-206
        ("ref_decode", 2, 2, 1, 7, 4, 3),       # cpu.rs:208-224
        ("ref_gqa", 4, 2, 6, 6, 4, 4),          # cpu.rs:226-242
        ("c1_decode", 14, 2, 1, 77, 64, 16),    # C1 heads, partial last page
        ("c1_prefix_prefill", 14, 2, 9, 40, 64, 16),
        ("llama_decode", 32, 8, 1, 20, 128, 16),
    ]
    for name, h, hkv, sq, kv, d, bs in specs:
        q = rng.uniform(-1, 1, (h, sq, d)).astype(np.float32)
        k = rng.uniform(-1, 1, (hkv, kv, d)).astype(np.float32)
        v = rng.uniform(-1, 1, (hkv, kv, d)).astype(np.float32)
        scale = 1.0 / np.sqrt(d)
        out = dense_f64(q, k, v, h // hkv, scale)
        cases[name] = dict(q=q, k=k, v=v, out=out.astype(np.float32), n_rep=np.int32(h // hkv),
                           scale=np.float64(scale), block_size=np.int32(bs))
    return cases


def main() -> None:
    (HERE / "reference_literals.json").write_text(json.dumps(literals(), indent=1) + "\n")
    cases = dense_cases(np.random.default_rng(20261201))
    flat = {f"{name}/{key}": val for name, c in cases.items() for key, val in c.items()}
    np.savez_compressed(HERE / "dense_f64_cases.npz", **flat)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
