"""Parity report: max-abs difference between the CUDA path and the oracle restatement of
src/backend/cpu.rs:57-112, per configuration, per score flow and per seed. Needs a GPU.

Rows: the default kernel flow (FA_SCORES_F32) against the oracle's f32 scores (score_mode 0);
the reference flow (FA_SCORES_REFERENCE) against the oracle's restatement of the reference's
bf16 dtype flow (score_mode 1, cpu.rs:84-85); and, for information, the default kernel flow
against that reference flow (how far f32 scores sit from the reference's rounding).

    python tests/parity_report.py [--seeds 3] [--json out.json]

Sizes: C1 whole; C2 all 64 sequences (one layer); C3 whole (one layer); C4 4 sequences of
16K-32K tokens; C5 decode 64 sequences of its context distribution and C5 prefill 8 prompts of
L ~ U[256, 2048] (Qwen2-7B heads). Not collected by pytest (no test_ prefix): the tests assert
the bound, this script reports the numbers behind it.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from flour_b200 import ops  # noqa: E402
from flour_b200.workloads import (LLAMA8B, QWEN7B, c2_contexts, c4_contexts,  # noqa: E402
                                  c5_contexts, make_c1, make_c3, make_decode, make_prefill)
from _util import f32, oracle_attention  # noqa: E402


def decode_case(b, flow):
    h = b.heads
    out = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens,
                           h.n_rep, 1 / math.sqrt(h.head_dim), b.max_context_len,
                           ops.Workspace(b.q.device), score_flow=flow)
    cu = torch.arange(b.num_seqs + 1, dtype=torch.int32)
    return out, cu, b.context_lens


def prefill_case(b, flow):
    h = b.heads
    ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    out = ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                            b.block_tables, h.n_rep, 1 / math.sqrt(h.head_dim), b.max_seqlen_q,
                            b.max_context_len, ops.Workspace(b.q.device), score_flow=flow)
    return out, b.cu_seqlens_q, b.context_lens


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seeds", type=int, default=3)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    cases = {
        "C1 (f32, decode)": lambda s: (decode_case, make_c1(dev, seed=s)),
        "C2 (bf16, decode, 64 seqs)": lambda s: (decode_case, make_decode(
            LLAMA8B, c2_contexts(s), torch.bfloat16, dev, s)),
        "C3 (bf16, prefill, full)": lambda s: (prefill_case, make_c3(dev, seed=s)),
        "C4 (bf16, decode, 4 x 16K-32K)": lambda s: (decode_case, make_decode(
            LLAMA8B, c4_contexts(s, 4), torch.bfloat16, dev, s)),
        "C5 decode (bf16, 64 seqs)": lambda s: (decode_case, make_decode(
            QWEN7B, c5_contexts(s, 64), torch.bfloat16, dev, s)),
        "C5 prefill (bf16, 8 prompts)": lambda s: (prefill_case, make_prefill(
            QWEN7B, np.random.default_rng(s).integers(256, 2049, size=8), np.zeros(8, np.int64),
            torch.bfloat16, dev, s)),
    }
    rows = []
    combos = ((0, 0, "kernel f32 vs oracle f32"), (1, 1, "kernel reference vs oracle reference"),
              (0, 1, "kernel f32 vs oracle reference (info)"))
    for name, make in cases.items():
        for k in range(a.seeds):
            seed = 2000 + 17 * k
            run, b = make(seed)
            h = b.heads
            outs, want = {}, {}
            for flow in (0, 1):
                out, cu, ctx = run(b, flow)
                torch.cuda.synchronize()
                assert ops.device_status() == 0
                outs[flow] = f32(out).astype(np.float64)
                want[flow] = oracle_attention(b.q, b.k_caches[0], b.v_caches[0], cu, ctx,
                                              b.block_tables, h.n_rep, 1 / math.sqrt(h.head_dim),
                                              score_mode=flow)
            for kf, om, label in combos:
                d = np.abs(outs[kf] - want[om])
                rows.append({"config": name, "check": label, "seed": seed,
                             "max_abs": float(d.max()), "mean_abs": float(d.mean()),
                             "max_ref": float(np.abs(want[om]).max())})
            del b
            torch.cuda.empty_cache()
    print("| config | check | max-abs per seed | mean-abs | max abs(out) |")
    print("|---|---|---|---|---|")
    for name in cases:
        for _, _, label in combos:
            r = [x for x in rows if x["config"] == name and x["check"] == label]
            print(f"| {name} | {label} | " + ", ".join(f"{x['max_abs']:.2e}" for x in r)
                  + f" | {np.mean([x['mean_abs'] for x in r]):.1e} | "
                  f"{max(x['max_ref'] for x in r):.2f} |")
    if a.json:
        Path(a.json).write_text(json.dumps(rows, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
