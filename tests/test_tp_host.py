"""Host logic of the head-sharded decode group, on CPU (gloo, world_size 2).

  * head_shard: which KV / query heads each rank holds, and its errors;
  * the output contract the kernel implements (rank r's head outputs land at head offset
    r * num_heads/tp of every rank's buffer), restated with the oracle: each rank decodes its
    head shard only, places it into a full-size buffer, and the buffers exchanged over gloo
    assemble into exactly the single-rank output, bit for bit;
  * HeadShardedGroup's handle exchange and the fa_tp_group it builds (buffer offsets by decode
    parity, peers' flag arrays, own epoch counter), with a stand-in for the C library's IPC
    calls so no GPU is needed.
"""

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

from flour_b200 import FlourAttnError
from flour_b200.tp import HeadShardedGroup, head_shard

WORLD = 2


def test_head_shard():
    assert head_shard(32, 8, 2, 0) == (0, 4, 0, 16)
    assert head_shard(32, 8, 2, 1) == (4, 8, 16, 32)
    assert head_shard(28, 4, 4, 3) == (3, 4, 21, 28)
    assert head_shard(14, 2, 1, 0) == (0, 2, 0, 14)
    for args in [(32, 8, 3, 0), (32, 8, 2, 2), (32, 8, 0, 0), (30, 8, 2, 0), (64, 16, 9, 0)]:
        with pytest.raises(FlourAttnError):
            head_shard(*args)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem():
    import oracle
    rng = np.random.default_rng(77)
    ctx = rng.integers(1, 200, size=6).astype(np.int32)
    hq, hkv, d, bs = 8, 4, 32, 16
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
    return q, kc, vc, ctx, bt


def decode(q, kc, vc, ctx, bt, n_rep):
    import oracle
    out, err = oracle.paged_attention(q, kc, vc, np.arange(len(ctx) + 1, dtype=np.int32), ctx, bt,
                                      n_rep, 1 / np.sqrt(q.shape[-1]), dtype=oracle.DT_BF16,
                                      threads=1)
    assert err == 0
    return out


class FakeIpc:
    """Stand-in for the library's IPC calls: rank r's allocation sits at (r + 1) << 40 and a
    handle names it; opening a peer's handle maps it at base + (1 << 36)."""

    def __init__(self, rank):
        self.rank, self.closed, self.freed = rank, [], []

    def fa_ipc_alloc(self, nbytes, ptr_ref, handle_ref):
        self.nbytes = nbytes
        ptr_ref._obj.value = (self.rank + 1) << 40
        handle_ref._obj.bytes[:8] = list(((self.rank + 1) << 40).to_bytes(8, "little"))
        return 0

    def fa_ipc_open(self, handle_ref, ptr_ref):
        ptr_ref._obj.value = int.from_bytes(bytes(handle_ref._obj.bytes[:8]), "little") + (1 << 36)
        return 0

    def fa_ipc_close(self, ptr):
        self.closed.append(ptr.value)
        return 0

    def fa_ipc_free(self, ptr):
        self.freed.append(ptr.value)
        return 0


def worker(rank, port, results):
    try:
        import torch.distributed as dist
        from flour_b200.tp import torch_exchange
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=20))
        # (1) the output contract, with the oracle as the decode.
        q, kc, vc, ctx, bt = problem()
        kv0, kv1, h0, h1 = head_shard(q.shape[1], kc.shape[1], WORLD, rank)
        mine = decode(np.ascontiguousarray(q[:, h0:h1]), np.ascontiguousarray(kc[:, kv0:kv1]),
                      np.ascontiguousarray(vc[:, kv0:kv1]), ctx, bt, q.shape[1] // kc.shape[1])
        buf = np.zeros_like(q)
        buf[:, h0:h1] = mine
        bufs = [None] * WORLD
        dist.all_gather_object(bufs, buf)
        assembled = np.zeros_like(q)
        for r in range(WORLD):
            _, _, a, b = head_shard(q.shape[1], kc.shape[1], WORLD, r)
            assembled[:, a:b] = bufs[r][:, a:b]
        full = decode(q, kc, vc, ctx, bt, q.shape[1] // kc.shape[1])
        contract_ok = bool(np.array_equal(assembled, full))
        # (2) the group's handle exchange and fa_tp_group, without a GPU.
        fake = FakeIpc(rank)
        grp = HeadShardedGroup(WORLD, rank, 10, 32, 128, torch.bfloat16, torch_exchange(),
                               device="cpu", lib=fake)
        lay = grp.layout
        groups = {}
        for epoch in (1, 2):
            g = grp.group_for(epoch)
            groups[epoch] = (g.tp, g.rank, [g.out[r] for r in range(WORLD)],
                             [g.flags[r] for r in range(WORLD)], g.epoch_counter)
        grp.close()
        results.put((rank, "ok", (contract_ok, fake.nbytes, lay.stride, lay.flags_off,
                                  lay.epoch_off, groups, fake.closed, fake.freed)))
        dist.destroy_process_group()
    except Exception as e:
        results.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


def test_group_host_logic_two_ranks():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        rank, kind, payload = results.get(timeout=120)
        out[rank] = (kind, payload)
    for p in procs:
        p.join(timeout=30)
    base = lambda r: (r + 1) << 40
    mapped = lambda r, me: base(r) if r == me else base(r) + (1 << 36)
    for rank, (kind, payload) in out.items():
        assert kind == "ok", f"rank {rank}: {payload}"
        contract_ok, nbytes, stride, flags_off, epoch_off, groups, closed, freed = payload
        assert contract_ok, f"rank {rank}: assembled head shards differ from the full decode"
        out_bytes = 10 * 32 * 128 * 2
        assert stride == (out_bytes + 255) // 256 * 256 and flags_off == 2 * stride
        assert epoch_off == flags_off + 256 and nbytes == epoch_off + 256
        for epoch, (tp, grank, outs, flags, epoch_counter) in groups.items():
            assert (tp, grank) == (WORLD, rank)
            off = 0 if epoch % 2 else stride  # odd epochs use the first buffer
            assert outs == [mapped(r, rank) + off for r in range(WORLD)]
            assert flags == [mapped(r, rank) + flags_off for r in range(WORLD)]
            assert epoch_counter == base(rank) + epoch_off
        assert closed == [mapped(r, rank) for r in range(WORLD) if r != rank]
        assert freed == [base(rank)]
