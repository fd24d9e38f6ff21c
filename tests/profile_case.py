"""Profiling fixture: small, fixed cases for Nsight Compute captures of one kernel.

    python tests/profile_case.py decode  [--launches 3] [--batch 64] [--seed 1000]
    python tests/profile_case.py longctx [--launches 3]
    python tests/profile_case.py prefill [--launches 3]
    python tests/profile_case.py qkv     [--launches 3] [--tokens 13490]
    python tests/profile_case.py oproj   [--launches 3] [--tokens 13490]
    python tests/profile_case.py bundle  [--launches 3]

Not collected by pytest (no test_ prefix); the profiles/*.md summaries name the command line
that made them.

`decode` is one layer of the C2 configuration (64 sequences, ctx ~ U[512, 4096], ~0.6 GB of
KV: larger than L2, a few GB at most on the device). `longctx` is 4 sequences of the C4
distribution (split-K heavy). `prefill` is one layer of C3. Each case runs one warm-up launch
and then `--launches` launches of the kernel under test, and exits 0. `qkv` / `oproj` are the
fused Llama-3-8B projections (hidden 4096) at `--tokens` tokens (13490 = one C3 batch: the
activations and weights exceed L2).
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from flour_b200 import ops  # noqa: E402
from flour_b200.workloads import LLAMA8B, c2_contexts, c4_contexts, make_c3, make_decode


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["decode", "longctx", "prefill", "qkv", "oproj", "bundle"])
    ap.add_argument("--tokens", type=int, default=13490)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seed", type=int, default=1000)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    scale = 1.0 / math.sqrt(128)
    if a.case in ("decode", "longctx"):
        ctx = c2_contexts(a.seed, a.batch) if a.case == "decode" else c4_contexts(a.seed, 4)
        b = make_decode(LLAMA8B, ctx, torch.bfloat16, dev, a.seed)
        ws = ops.Workspace(dev)
        out = torch.empty_like(b.q)
        for _ in range(1 + a.launches):
            ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens, 4,
                             scale, b.max_context_len, ws, out=out)
        torch.cuda.synchronize()
        print(f"{a.case}: {b.kv_bytes_per_layer() + b.io_bytes_per_layer()} algorithmic bytes/launch")
    elif a.case in ("qkv", "oproj"):
        from flour_b200.paged import rope_tables
        T, hidden, hq, hkv, d = a.tokens, 4096, 32, 8, 128
        g = torch.Generator(device=dev).manual_seed(a.seed)
        x = torch.randn(T, hidden, device=dev, generator=g).to(torch.bfloat16)
        if a.case == "qkv":
            n = (hq + 2 * hkv) * d
            w = (torch.randn(n, hidden, device=dev, generator=g) / 64).to(torch.bfloat16)
            kc = torch.zeros(T // 16 + 8, hkv, 16, d, device=dev, dtype=torch.bfloat16)
            vc = torch.zeros_like(kc)
            pos = torch.arange(T, dtype=torch.int32, device=dev) % 8192
            slots = torch.arange(T, dtype=torch.int32, device=dev)
            cos, sin = rope_tables(d, 8192, 500000.0, torch.bfloat16, dev)
            q = torch.empty(T, hq, d, device=dev, dtype=torch.bfloat16)
            for _ in range(1 + a.launches):
                ops.qkv_rope_cache(x, w, kc, vc, pos, slots, hq, cos, sin, q_out=q)
            flops = 2 * T * hidden * n
        else:
            w = (torch.randn(hidden, hq * d, device=dev, generator=g) / 64).to(torch.bfloat16)
            attn = torch.randn(T, hq * d, device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty(T, hidden, device=dev, dtype=torch.bfloat16)
            for _ in range(1 + a.launches):
                ops.o_proj_residual(attn, w, x, out=out)
            flops = 2 * T * hq * d * hidden
        torch.cuda.synchronize()
        print(f"{a.case}: {flops} algorithmic FLOPs/launch")
    elif a.case == "bundle":
        # FLKV export of 128 blocks x 32 layers (Llama-3-8B heads, 268 MB payload) from 32 pools
        # of 512 blocks (1 GB): the one-launch gather.
        import numpy as np
        g = torch.Generator(device=dev).manual_seed(a.seed)
        ks = [torch.randn((512, 8, 16, 128), device=dev, generator=g).to(torch.bfloat16)
              for _ in range(32)]
        vs = [torch.randn((512, 8, 16, 128), device=dev, generator=g).to(torch.bfloat16)
              for _ in range(32)]
        ids = torch.from_numpy(np.random.default_rng(a.seed).permutation(512)[:128].astype(np.int32)
                               ).to(dev)
        payload = torch.empty(ops.bundle_payload_bytes(ks, vs, 128), dtype=torch.uint8, device=dev)
        for _ in range(1 + a.launches):
            ops.export_bundle_payload(ks, vs, ids, payload)
        torch.cuda.synchronize()
        print(f"bundle: {2 * payload.numel()} algorithmic bytes/launch (read + write)")
    else:
        b = make_c3(dev, seed=a.seed)
        ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
        ws = ops.Workspace(dev)
        out = torch.empty_like(b.q)
        for _ in range(1 + a.launches):
            ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                              b.block_tables, 4, scale, b.max_seqlen_q, b.max_context_len, ws,
                              out=out)
        torch.cuda.synchronize()
        print(f"prefill: {b.flops()} algorithmic FLOPs/launch")
    st = ops.device_status()
    if st:
        raise SystemExit(f"device status 0x{st:x}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
