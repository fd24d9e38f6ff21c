"""Sequence sharding across ranks, on CPU with the gloo backend (world_size 2).

Every rank derives the same seeded batch, takes its LPT shard of the sequences, runs the oracle
on that shard only, and the shards are gathered: together they must equal the single-rank
result bit for bit and cover every sequence exactly once (no collective is needed on the data
path; the gather here is only the test's checker). A second case has one rank fail before the
exchange: the surviving rank must see an error from the collective instead of hanging.
"""

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np

WORLD = 2


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem():
    import oracle
    from flour_b200.workloads import c5_contexts
    rng = np.random.default_rng(55)
    ctx = c5_contexts(55, n=24) // 8 + 1  # C5's lognormal shape, shortened for a CPU test
    hq, hkv, d, bs = 28, 4, 32, 16
    pages = (ctx + bs - 1) // bs
    perm = rng.permutation(int(pages.sum())).astype(np.int32)
    bt = np.zeros((len(ctx), int(pages.max())), np.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n]
        o += n
    kc = oracle.f32_to_bf16(rng.standard_normal((len(perm), hkv, bs, d)).astype(np.float32))
    vc = oracle.f32_to_bf16(rng.standard_normal((len(perm), hkv, bs, d)).astype(np.float32))
    q = oracle.f32_to_bf16(rng.standard_normal((len(ctx), hq, d)).astype(np.float32))
    return q, kc, vc, ctx.astype(np.int32), bt


def run_shard(idx, q, kc, vc, ctx, bt):
    import oracle
    idx = np.asarray(idx, dtype=np.int64)
    out, err = oracle.paged_attention(q[idx], kc, vc, np.arange(len(idx) + 1, dtype=np.int32),
                                      ctx[idx], bt[idx], 7, 1 / np.sqrt(32),
                                      dtype=oracle.DT_BF16, threads=1)
    assert err == 0
    return out


def worker(rank, port, fail_rank, results):
    try:
        import torch.distributed as dist
        from flour_b200.workloads import lpt_partition
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=20))
        q, kc, vc, ctx, bt = problem()
        parts = lpt_partition(ctx, WORLD)
        mine = parts[rank]
        out = run_shard(mine, q, kc, vc, ctx, bt)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the exchange")
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (mine, out))
        results.put((rank, "ok", gathered))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides pass/fail
        results.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def launch(fail_rank):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, port, fail_rank, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        r, status, payload = results.get(timeout=120)
        got[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return got


def test_sequence_sharding_matches_single_rank():
    got = launch(fail_rank=-1)
    assert all(s == "ok" for s, _ in got.values()), got
    gathered = got[0][1]
    q, kc, vc, ctx, bt = problem()
    full = run_shard(np.arange(len(ctx)), q, kc, vc, ctx, bt)
    seen = np.zeros(len(ctx), dtype=int)
    for idx, out in gathered:
        seen[idx] += 1
        np.testing.assert_array_equal(out, full[np.asarray(idx)])
    assert (seen == 1).all()


def test_failed_rank_surfaces_as_error_not_hang():
    got = launch(fail_rank=1)
    assert got[1][0] == "error" and "injected" in got[1][1]
    assert got[0][0] == "error", got[0]
