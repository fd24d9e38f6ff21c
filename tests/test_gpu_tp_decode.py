"""Head-sharded decode (fa_paged_decode_tp + fa_tp_sync) on the GPU.

The kernel writes each rank's head outputs into every rank's output buffer; fa_tp_sync publishes
an epoch flag to every rank and waits for all of them, after which every rank holds the full
decode output. Checked here:
  * tp = 1 through HeadShardedGroup: bit-identical to fa_paged_decode (same kernel, same plan),
    over several epochs (both output buffers of the parity scheme);
  * tp = 2 and 4 emulated in one process on one GPU (every rank's buffers local; all decodes and
    publishes run one after the other on one stream before any wait, so no launch waits for a
    later one): every rank's buffer equals the oracle, including a sequence with an empty context
    (zeros + FA_DEVERR_CONTEXT);
  * a wait for a rank that never publishes ends after its time limit with FA_DEVERR_TIMEOUT and
    leaves the context usable;
  * with >= 2 GPUs: two processes, one GPU each, buffers mapped with CUDA IPC, the stores cross
    NVLink (skipped on a one-GPU box).
"""

import ctypes
import math
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

from flour_b200 import _lib, ops
from flour_b200.tp import HeadShardedGroup, head_shard
from flour_b200.workloads import LLAMA8B, QWEN7B, c2_contexts, make_decode

from _util import f32, max_abs, oracle_attention

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def shard_batch(b, tp, rank):
    """This rank's slice of a decode batch: its KV heads of the pool, its query heads."""
    h = b.heads
    kv0, kv1, h0, h1 = head_shard(h.num_heads, h.num_kv_heads, tp, rank)
    return (b.q[:, h0:h1].contiguous(), b.k_caches[0][:, kv0:kv1].contiguous(),
            b.v_caches[0][:, kv0:kv1].contiguous())


def full_oracle(b):
    h = b.heads
    cu = torch.arange(b.num_seqs + 1, dtype=torch.int32)
    return oracle_attention(b.q, b.k_caches[0], b.v_caches[0], cu, b.context_lens, b.block_tables,
                            h.n_rep, 1.0 / math.sqrt(h.head_dim))


def test_tp1_group_matches_single_gpu_decode(device):
    h = LLAMA8B
    grp = HeadShardedGroup(1, 0, 16, h.num_heads, h.head_dim, torch.bfloat16, lambda x: [x], device)
    try:
        ws = ops.Workspace(device)
        for epoch, seed in enumerate([5, 6, 7], start=1):
            b = make_decode(h, c2_contexts(seed, batch=16), torch.bfloat16, device, seed)
            scale = 1.0 / math.sqrt(h.head_dim)
            want = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                    b.context_lens, h.n_rep, scale, b.max_context_len, ws)
            got = grp.decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens,
                             h.n_rep, scale, b.max_context_len, ws)
            torch.cuda.synchronize()
            assert grp.epoch == epoch
            assert ops.device_status() == 0
            assert torch.equal(got, want), f"epoch {epoch}: differs from fa_paged_decode"
    finally:
        torch.cuda.synchronize()
        grp.close()


def test_tp_group_replays_in_a_cuda_graph(device):
    # Device-counted epochs: two captured decode calls (one per output buffer) replayed three
    # times with new queries; each replay's outputs equal fa_paged_decode's.
    h = LLAMA8B
    b = make_decode(h, c2_contexts(21, batch=8), torch.bfloat16, device, 21)
    scale = 1.0 / math.sqrt(h.head_dim)
    grp = HeadShardedGroup(1, 0, 8, h.num_heads, h.head_dim, torch.bfloat16, lambda x: [x], device)
    try:
        ws = ops.Workspace(device)
        ws.get(ops.workspace_size(8, h.num_heads, h.num_kv_heads, h.head_dim, b.max_context_len, 1))
        q1, q2 = b.q.clone(), b.q.clone()
        args = (b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens, h.n_rep, scale,
                b.max_context_len, ws)
        grp.decode(q1, *args)  # eager warm-up
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o1 = grp.decode(q1, *args)
            o2 = grp.decode(q2, *args)
        assert o1.data_ptr() != o2.data_ptr()
        gen = torch.Generator(device=device).manual_seed(3)
        for _ in range(3):
            q1.copy_(torch.randn(q1.shape, device=device, generator=gen))
            q2.copy_(torch.randn(q2.shape, device=device, generator=gen))
            graph.replay()
            torch.cuda.synchronize()
            assert ops.device_status() == 0
            assert torch.equal(o1, ops.paged_decode(q1, *args))
            assert torch.equal(o2, ops.paged_decode(q2, *args))
        del graph
    finally:
        torch.cuda.synchronize()
        grp.close()


def local_groups(tp, num_seqs, num_heads, head_dim, device):
    """tp groups whose buffers all live on this GPU (rank r's out and flags tensors)."""
    outs = [torch.zeros((num_seqs, num_heads, head_dim), dtype=torch.bfloat16, device=device)
            for _ in range(tp)]
    flags = [torch.zeros(_lib.FA_MAX_TP, dtype=torch.int32, device=device) for _ in range(tp)]
    groups = []
    for rank in range(tp):
        g = _lib.FaTpGroup()
        g.tp, g.rank = tp, rank
        for r in range(tp):
            g.out[r] = outs[r].data_ptr()
            g.flags[r] = flags[r].data_ptr()
        groups.append(g)
    return groups, outs, flags


@pytest.mark.parametrize("tp,heads", [(2, LLAMA8B), (4, LLAMA8B), (4, QWEN7B)])
def test_tp_emulated_on_one_gpu(device, tp, heads):
    h = heads
    b = make_decode(h, c2_contexts(40 + tp, batch=12), torch.bfloat16, device, 40 + tp)
    cl = b.context_lens.clone()
    cl[3] = 0  # empty context: zero output, FA_DEVERR_CONTEXT, flags still published
    groups, outs, flags = local_groups(tp, b.num_seqs, h.num_heads, h.head_dim, device)
    lib = _lib.lib()
    scale = 1.0 / math.sqrt(h.head_dim)
    ws = [ops.Workspace(device) for _ in range(tp)]
    stream = ops._stream()
    for epoch in (1, 2):
        for rank in range(tp):
            q, kc, vc = shard_batch(b, tp, rank)
            layer = ops.layer_desc(kc, vc)
            need = ops.workspace_size(b.num_seqs, q.shape[1], kc.shape[1], h.head_dim,
                                      b.max_context_len, 1)
            wp, wn = ops._ws_args(ws[rank], need)
            _lib.check(lib.fa_paged_decode_tp(ctypes.byref(groups[rank]), ctypes.byref(layer),
                                              ops._ptr(q), ops._ptr(cl),
                                              ops._ptr(b.block_tables), b.block_tables.shape[1],
                                              b.num_seqs, q.shape[1], h.n_rep, b.max_context_len,
                                              scale, 0, wp, wn, stream), "paged_decode_tp")
            _lib.check(lib.fa_tp_sync(ctypes.byref(groups[rank]), epoch, _lib.FA_TP_PUBLISH, 0,
                                      stream), "tp_sync publish")
        for rank in range(tp):
            _lib.check(lib.fa_tp_sync(ctypes.byref(groups[rank]), epoch, _lib.FA_TP_WAIT,
                                      10_000_000, stream), "tp_sync wait")
        torch.cuda.synchronize()
        status = ops.device_status()
        assert status == _lib.FA_DEVERR_CONTEXT, hex(status)
        for r in range(tp):
            assert flags[r][:tp].tolist() == [epoch] * tp
    want = full_oracle(b)
    keep = [i for i in range(b.num_seqs) if i != 3]
    for r in range(tp):
        err = max_abs(f32(outs[r])[keep], want[keep])
        assert err <= TOL_BF16, f"rank {r}: max-abs {err}"
        assert torch.equal(outs[r], outs[0])
        assert not outs[r][3].any()


def test_wait_times_out_and_context_survives(device):
    # Rank 0 of an emulated pair publishes and waits; rank 1 never publishes, so the wait ends
    # after its 1 ms limit with FA_DEVERR_TIMEOUT. The context stays usable afterwards.
    h = LLAMA8B
    groups, *_ = local_groups(2, 4, h.num_heads, h.head_dim, device)
    lib = _lib.lib()
    assert ops.device_status() == 0
    _lib.check(lib.fa_tp_sync(ctypes.byref(groups[0]), 1, _lib.FA_TP_PUBLISH | _lib.FA_TP_WAIT,
                              1_000_000, ops._stream()), "tp_sync")
    torch.cuda.synchronize()
    assert ops.device_status() == _lib.FA_DEVERR_TIMEOUT
    b = make_decode(h, np.array([100, 2000, 17, 5]), torch.bfloat16, device, 3)
    grp = HeadShardedGroup(1, 0, 4, h.num_heads, h.head_dim, torch.bfloat16, lambda x: [x], device)
    try:
        got = grp.decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens,
                         h.n_rep, 1.0 / math.sqrt(h.head_dim), b.max_context_len,
                         ops.Workspace(device))
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert max_abs(f32(got), full_oracle(b)) <= TOL_BF16
    finally:
        torch.cuda.synchronize()
        grp.close()


def test_tp_rejects_bad_groups_and_unsynced_decodes(device):
    h = LLAMA8B
    groups, *_ = local_groups(2, 4, h.num_heads, h.head_dim, device)
    lib = _lib.lib()
    g = groups[0]
    both = _lib.FA_TP_PUBLISH | _lib.FA_TP_WAIT
    g.rank = 2
    assert lib.fa_tp_sync(ctypes.byref(g), 1, both, 1_000_000, None) == _lib.FA_EINVAL
    g.rank = 0
    assert lib.fa_tp_sync(ctypes.byref(g), 0, both, 1_000_000, None) == _lib.FA_EINVAL  # no counter
    assert lib.fa_tp_sync(ctypes.byref(g), 1, both, 10, None) == _lib.FA_ERANGE
    assert lib.fa_tp_sync(ctypes.byref(g), 1, 4, 1_000_000, None) == _lib.FA_EINVAL
    g.out[1] = None
    b = make_decode(h, np.array([64]), torch.bfloat16, device, 1)
    q, kc, vc = shard_batch(b, 2, 0)
    layer = ops.layer_desc(kc, vc)
    st = lib.fa_paged_decode_tp(ctypes.byref(g), ctypes.byref(layer), ops._ptr(q),
                                ops._ptr(b.context_lens), ops._ptr(b.block_tables), 4, 1,
                                q.shape[1], h.n_rep, 64, 0.1, 0, None, 0, None)
    assert st == _lib.FA_EINVAL
    assert b"out[1]" in lib.fa_last_error_message()
    grp = HeadShardedGroup(1, 0, 1, h.num_heads, h.head_dim, torch.bfloat16, lambda x: [x], device)
    try:
        args = (b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens, h.n_rep, 0.1, 64,
                ops.Workspace(device))
        grp.decode(b.q, *args, wait=False)
        with pytest.raises(_lib.FlourAttnError):
            grp.decode(b.q, *args)  # the first decode was not synced
        grp.sync()
        grp.decode(b.q, *args)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
    finally:
        torch.cuda.synchronize()
        grp.close()


# ---- two processes, one GPU each, CUDA IPC over NVLink ----------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ipc_worker(rank, tp, port, results):
    try:
        import torch.distributed as dist
        from flour_b200.tp import torch_exchange
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=tp, timeout=timedelta(seconds=60))
        h = LLAMA8B
        grp = HeadShardedGroup(tp, rank, 32, h.num_heads, h.head_dim, torch.bfloat16,
                               torch_exchange(), dev)
        ws = ops.Workspace(dev)
        errs = []
        for seed in (11, 12, 13):
            b = make_decode(h, c2_contexts(seed, batch=32), torch.bfloat16, dev, seed)
            q, kc, vc = shard_batch(b, tp, rank)
            got = grp.decode(q, kc, vc, b.block_tables, b.context_lens, h.n_rep,
                             1.0 / math.sqrt(h.head_dim), b.max_context_len, ws)
            torch.cuda.synchronize()
            status = ops.device_status()
            full = ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                    b.context_lens, h.n_rep, 1.0 / math.sqrt(h.head_dim),
                                    b.max_context_len, ws)
            errs.append((status, max_abs(f32(got), full_oracle(b)), max_abs(f32(got), f32(full))))
        dist.barrier()  # every rank's stores into the others' buffers are done
        grp.close()
        dist.destroy_process_group()
        results.put((rank, "ok", errs))
    except Exception as e:
        results.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


def test_tp2_two_processes_ipc():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    tp = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ipc_worker, args=(r, tp, port, results)) for r in range(tp)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(tp):
        rank, kind, payload = results.get(timeout=300)
        out[rank] = (kind, payload)
    for p in procs:
        p.join(timeout=60)
    for rank, (kind, payload) in out.items():
        assert kind == "ok", f"rank {rank}: {payload}"
        for status, err_oracle, err_single in payload:
            assert status == 0
            assert err_oracle <= TOL_BF16
            assert err_single <= TOL_BF16
