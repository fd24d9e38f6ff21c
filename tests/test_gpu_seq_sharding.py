"""Sequence sharding on two GPUs: one process per GPU, NCCL process group (the bench's layout).
Every rank builds the same seeded C5-style decode batch and prompt set (Qwen2-7B heads), runs
the decode and the prefill on its own share of the sequences only (workloads.mixed_partition,
the partition bench.py uses), and the shares are gathered over NCCL for the check: together
they must cover every sequence once and match the single-GPU results for the whole batch (which
the oracle tests cover) within a bf16 ulp, the split-K plan being chosen per batch size. No
collective is on the data path itself; the gather is the test's checker. Skips with fewer than
two GPUs."""

import math
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2
TOL = 1.6e-2  # one bf16 ulp at |out| in [2, 4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, results):
    try:
        import torch.distributed as dist
        from flour_b200 import ops
        from flour_b200.workloads import (QWEN7B, c5_plan, make_decode, make_prefill,
                                          mixed_partition)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                                timeout=timedelta(seconds=120), device_id=dev)
        h = QWEN7B
        scale = 1 / math.sqrt(h.head_dim)
        ctx, is_pf, pf_len, cost = c5_plan(90, n=96)
        ctx = np.minimum(ctx, 3000)
        shares = mixed_partition(cost, is_pf, WORLD)
        dec_all = [i for i in range(len(ctx)) if not is_pf[i]]
        pf_all = [i for i in range(len(ctx)) if is_pf[i]][:6]
        # The whole batch (same seed on every rank), and this rank's share of it.
        full_dec = make_decode(h, ctx[dec_all], torch.bfloat16, dev, 91)
        full_pf = make_prefill(h, pf_len[pf_all], np.zeros(len(pf_all), np.int64), torch.bfloat16,
                               dev, 92)
        mine = set(shares[rank])
        d_idx = [k for k, i in enumerate(dec_all) if i in mine]
        p_idx = [k for k, i in enumerate(pf_all) if i in mine]
        ws = ops.Workspace(dev)
        b = full_dec
        idx = torch.tensor(d_idx, dtype=torch.long, device=dev)
        dec_out = ops.paged_decode(b.q[idx].contiguous(), b.k_caches[0], b.v_caches[0],
                                   b.block_tables[idx].contiguous(),
                                   b.context_lens[idx].contiguous(), h.n_rep, scale,
                                   int(b.ctx_host[d_idx].max()) if d_idx else 1, ws)
        # Prefill share: the prompts' packed rows, re-packed for this rank's sequences.
        p = full_pf
        ops.reshape_and_cache(p.k_caches[0], p.v_caches[0], p.key, p.value, p.slot_mapping)
        cu = p.cu_seqlens_q.cpu().numpy()
        rows = np.concatenate([np.arange(cu[k], cu[k + 1]) for k in p_idx]) if p_idx else \
            np.zeros(0, np.int64)
        lens = np.array([cu[k + 1] - cu[k] for k in p_idx], dtype=np.int64)
        my_cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        rows_t = torch.tensor(rows, dtype=torch.long, device=dev)
        pf_out = None
        if p_idx:
            pf_out = ops.paged_prefill(p.q[rows_t].contiguous(), p.k_caches[0], p.v_caches[0],
                                       my_cu, p.context_lens[p_idx].contiguous(),
                                       p.block_tables[p_idx].contiguous(), h.n_rep, scale,
                                       int(lens.max()), int(lens.max()), ops.Workspace(dev))
        torch.cuda.synchronize()
        status = ops.device_status()
        # Checker: gather every rank's share (padded) to rank 0 over NCCL.
        def gather(t, n_rows, shape):
            buf = torch.zeros((n_rows,) + shape, dtype=torch.bfloat16, device=dev)
            if t is not None and t.shape[0]:
                buf[:t.shape[0]] = t
            parts = [torch.empty_like(buf) for _ in range(WORLD)]
            dist.all_gather(parts, buf)
            return parts
        n_dec = [len([i for i in dec_all if i in set(s)]) for s in shares]
        n_rows = [int(sum(cu[k + 1] - cu[k] for k, i in enumerate(pf_all) if i in set(s)))
                  for s in shares]
        dec_parts = gather(dec_out, max(n_dec), tuple(b.q.shape[1:]))
        pf_parts = gather(pf_out, max(max(n_rows), 1), tuple(p.q.shape[1:]))
        errs = None
        if rank == 0:
            want_dec = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                        b.context_lens, h.n_rep, scale, b.max_context_len, ws)
            want_pf = ops.paged_prefill(p.q, p.k_caches[0], p.v_caches[0], p.cu_seqlens_q,
                                        p.context_lens, p.block_tables, h.n_rep, scale,
                                        p.max_seqlen_q, p.max_context_len, ops.Workspace(dev))
            got_dec = torch.empty_like(want_dec)
            got_pf = torch.empty_like(want_pf)
            seen_dec, seen_rows = [], []
            for r, s in enumerate(shares):
                sd = [k for k, i in enumerate(dec_all) if i in set(s)]
                got_dec[torch.tensor(sd, dtype=torch.long, device=dev)] = dec_parts[r][:len(sd)]
                seen_dec += sd
                sp = [k for k, i in enumerate(pf_all) if i in set(s)]
                rr = np.concatenate([np.arange(cu[k], cu[k + 1]) for k in sp]) if sp else \
                    np.zeros(0, np.int64)
                got_pf[torch.tensor(rr, dtype=torch.long, device=dev)] = pf_parts[r][:len(rr)]
                seen_rows += list(rr)
            assert sorted(seen_dec) == list(range(len(dec_all)))
            assert sorted(seen_rows) == list(range(int(cu[-1])))
            errs = ((got_dec.float() - want_dec.float()).abs().max().item(),
                    (got_pf.float() - want_pf.float()).abs().max().item())
        dist.barrier()
        dist.destroy_process_group()
        results.put((rank, "ok", (status, errs, len(d_idx), len(p_idx))))
    except Exception as e:
        results.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-800:]}"))


def test_two_gpus_sequence_shards_match_single_gpu():
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        rank, kind, payload = results.get(timeout=600)
        out[rank] = (kind, payload)
    for p in procs:
        p.join(timeout=60)
    for rank, (kind, payload) in sorted(out.items()):
        assert kind == "ok", f"rank {rank}: {payload}"
        status, errs, n_dec, n_pf = payload
        assert status == 0
        assert n_dec > 0
    err_dec, err_pf = out[0][1][1]
    assert err_dec <= TOL and err_pf <= TOL, (err_dec, err_pf)
