"""Head-sharded decode: a layer's KV heads split over the GPUs of a group, one process per GPU.

The reference decodes on one CPU (src/backend/cpu.rs paged_attention, called from
src/models/common/attention.rs:104-109) and never shards heads; this optional mode exists for
models whose pool does not fit one GPU or whose per-token latency must drop below one GPU's.
Rank r holds KV heads [r*kv/tp, (r+1)*kv/tp) of every block and query heads
[r*hq/tp, (r+1)*hq/tp). ``fa_paged_decode_tp`` writes each rank's head outputs straight into
every rank's output buffer over NVLink (CUDA IPC mappings); ``fa_tp_sync`` then publishes an
epoch flag to every rank and makes the stream wait (bounded) for all ranks' flags. So after
``HeadShardedGroup.decode`` every rank holds the full [num_seqs, num_heads, head_dim] output
that a single-GPU decode produces, with no separate all-gather launch.

Memory of one rank (one cudaMalloc, one IPC handle; the same layout on every rank):
    [0, S)            output buffer of odd epochs   [max_seqs, num_heads, head_dim]
    [S, 2S)           output buffer of even epochs
    [2S, 2S+32)       flag array, FA_MAX_TP u32: slot s = last epoch rank s published here
    [2S+256, +4)      device epoch of this rank (advanced by each publish)
with S the output size rounded up to 256 bytes. Two output buffers alternate by decode parity so
that a rank one decode ahead never overwrites what a slower peer is still reading; this needs a
sync (publish + wait) after every decode, which ``decode`` does unless told not to, and then
``sync`` must come before the next ``decode``.

Epochs are counted on the device (``fa_tp_sync`` with epoch 0), so a sequence of ``decode``
calls can be captured in a CUDA graph and replayed; the host counts calls only to pick the
output buffer, so a captured sequence should hold an even number of calls.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import torch

from . import _lib
from ._lib import FA_MAX_TP, FA_TP_PUBLISH, FA_TP_WAIT, FaIpcHandle, FaTpGroup, FlourAttnError, check

DEFAULT_TIMEOUT_NS = 2_000_000_000


def head_shard(num_heads: int, num_kv_heads: int, tp: int, rank: int) -> tuple[int, int, int, int]:
    """(kv0, kv1, h0, h1): the KV heads and query heads rank `rank` of `tp` holds."""
    if tp < 1 or tp > FA_MAX_TP or not 0 <= rank < tp:
        raise FlourAttnError(_lib.FA_EINVAL, f"rank {rank} of tp {tp} (1..{FA_MAX_TP} ranks)")
    if num_kv_heads % tp or num_heads % num_kv_heads:
        raise FlourAttnError(_lib.FA_EINVAL,
                             f"num_kv_heads {num_kv_heads} must split evenly over {tp} ranks and "
                             f"divide num_heads {num_heads}")
    per = num_kv_heads // tp
    n_rep = num_heads // num_kv_heads
    kv0, kv1 = rank * per, (rank + 1) * per
    return kv0, kv1, kv0 * n_rep, kv1 * n_rep


def _r256(n: int) -> int:
    return (n + 255) // 256 * 256


class _Layout:
    def __init__(self, max_seqs: int, num_heads: int, head_dim: int, elem: int):
        self.out_bytes = max_seqs * num_heads * head_dim * elem
        self.stride = _r256(self.out_bytes)
        self.flags_off = 2 * self.stride
        self.epoch_off = self.flags_off + 256
        self.total = self.epoch_off + 256


class _CudaBytes:
    """A raw device range exposed through __cuda_array_interface__ so torch can view it."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


def torch_exchange(group=None) -> Callable[[object], list]:
    """An exchange function over torch.distributed: every rank's object, in rank order."""
    import torch.distributed as dist

    def exchange(obj):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, obj, group=group)
        return out
    return exchange


class HeadShardedGroup:
    """One rank's view of a head-sharded decode group.

    `exchange(obj) -> list` must return every rank's object in rank order (for example
    ``torch_exchange()``); it is called once, from the constructor, on all ranks together.
    `lib` is the loaded C library (tests pass a stand-in to check the host logic without a GPU).
    The group's buffers live until ``close()``; tensors returned by ``decode`` view them.
    """

    def __init__(self, tp: int, rank: int, max_seqs: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype, exchange: Callable[[object], Sequence], device=None,
                 lib=None):
        if tp < 1 or tp > FA_MAX_TP or not 0 <= rank < tp:
            raise FlourAttnError(_lib.FA_EINVAL, f"rank {rank} of tp {tp} (1..{FA_MAX_TP} ranks)")
        if dtype not in (torch.bfloat16, torch.float16):
            raise FlourAttnError(_lib.FA_EUNSUPPORTED, f"head-sharded decode needs bf16/f16, got {dtype}")
        if max_seqs < 1 or num_heads < 1 or head_dim < 1:
            raise FlourAttnError(_lib.FA_EINVAL, "max_seqs, num_heads and head_dim must be >= 1")
        self.tp, self.rank = tp, rank
        self.max_seqs, self.num_heads, self.head_dim, self.dtype = max_seqs, num_heads, head_dim, dtype
        self.device = torch.device(device if device is not None else "cuda")
        self._lib = lib if lib is not None else _lib.lib()
        self.layout = _Layout(max_seqs, num_heads, head_dim, torch.tensor([], dtype=dtype).element_size())
        self.epoch = 0          # decodes so far (= the device epoch once each is synced)
        self._pending = False   # a decode without its sync
        self._bases: list[int] = [0] * tp
        self._opened: list[int] = []
        ptr, handle = ctypes.c_void_p(), FaIpcHandle()
        check(self._lib.fa_ipc_alloc(self.layout.total, ctypes.byref(ptr), ctypes.byref(handle)),
              "ipc_alloc")
        self._local = int(ptr.value)
        self._bases[rank] = self._local
        try:
            handles = list(exchange(bytes(handle.bytes)))
            if len(handles) != tp:
                raise FlourAttnError(_lib.FA_EINVAL, f"exchange returned {len(handles)} handles for tp {tp}")
            for r, hb in enumerate(handles):
                if r == rank:
                    continue
                h = FaIpcHandle()
                ctypes.memmove(h.bytes, bytes(hb), 64)
                peer = ctypes.c_void_p()
                check(self._lib.fa_ipc_open(ctypes.byref(h), ctypes.byref(peer)), f"ipc_open(rank {r})")
                self._bases[r] = int(peer.value)
                self._opened.append(int(peer.value))
        except BaseException:
            self.close()
            raise
        self._groups = [self._make_group(parity) for parity in (0, 1)]
        self._views: list[torch.Tensor | None] = [None, None]

    def _make_group(self, parity: int) -> FaTpGroup:
        g = FaTpGroup()
        g.tp, g.rank = self.tp, self.rank
        off = (1 - parity) * self.layout.stride  # odd epochs use buffer 0
        for r in range(self.tp):
            g.out[r] = self._bases[r] + off
            g.flags[r] = self._bases[r] + self.layout.flags_off
        g.epoch_counter = self._local + self.layout.epoch_off
        return g

    def group_for(self, epoch: int) -> FaTpGroup:
        """The ``fa_tp_group`` (output buffers of this epoch's parity) of `epoch`."""
        return self._groups[epoch & 1]

    def output(self, epoch: int, num_seqs: int) -> torch.Tensor:
        """This rank's full output [num_seqs, num_heads, head_dim] of `epoch` (a view)."""
        parity = epoch & 1
        if self._views[parity] is None:
            base = self.group_for(epoch).out[self.rank]
            raw = torch.as_tensor(_CudaBytes(base, self.layout.out_bytes), device=self.device)
            self._views[parity] = raw.view(self.dtype).view(self.max_seqs, self.num_heads, self.head_dim)
        return self._views[parity][:num_seqs]

    def decode(self, query, k_cache, v_cache, block_tables, context_lens, n_rep: int, scale: float,
               max_context_len: int, workspace=None, wait: bool = True,
               timeout_ns: int = DEFAULT_TIMEOUT_NS, stream=None,
               score_flow: int = _lib.FA_SCORES_F32) -> torch.Tensor:
        """Decode this rank's heads (query [B, num_heads/tp, d], k/v_cache holding this rank's KV
        heads) into every rank's output and return the full [B, num_heads, d] output view. With
        `wait` (the default) the sync follows at once; otherwise call ``sync`` before reading the
        output or decoding again. Every rank makes the same calls."""
        from . import ops
        if self._pending:
            raise FlourAttnError(_lib.FA_EINVAL, "decode: the previous decode has not been synced")
        layer = ops.layer_desc(k_cache, v_cache)
        query = query.contiguous()
        B, hq, d = query.shape
        if B > self.max_seqs or hq * self.tp != self.num_heads or d != self.head_dim:
            raise FlourAttnError(_lib.FA_EINVAL,
                                 f"query {tuple(query.shape)} does not fit the group ({self.max_seqs} "
                                 f"seqs, {self.num_heads} heads over {self.tp} ranks, d {self.head_dim})")
        if query.dtype != self.dtype:
            raise FlourAttnError(_lib.FA_EINVAL, f"query dtype {query.dtype}, group dtype {self.dtype}")
        bt, cl = ops._i32(block_tables, "block_tables"), ops._i32(context_lens, "context_lens")
        need = ops.workspace_size(max(B, 1), hq, k_cache.shape[1], d, max(max_context_len, 1), 1)
        wp, wn = ops._ws_args(workspace, need)
        epoch = self.epoch + 1  # the device epoch its sync publishes (all ranks in lockstep)
        g = self.group_for(epoch)
        check(self._lib.fa_paged_decode_tp(ctypes.byref(g), ctypes.byref(layer), ops._ptr(query),
                                           ops._ptr(cl), ops._ptr(bt), bt.shape[1], B, hq, n_rep,
                                           max_context_len, scale, score_flow, wp, wn,
                                           ops._stream(stream)),
              "paged_decode_tp")
        self.epoch = epoch
        self._pending = True
        if wait:
            self.sync(timeout_ns, stream)
        return self.output(epoch, B)

    def sync(self, timeout_ns: int = DEFAULT_TIMEOUT_NS, stream=None) -> None:
        """Publish this rank's last decode to every rank and make `stream` wait (bounded) until
        every rank published it (device-counted epochs)."""
        from . import ops
        check(self._lib.fa_tp_sync(ctypes.byref(self._groups[0]), 0, FA_TP_PUBLISH | FA_TP_WAIT,
                                   timeout_ns, ops._stream(stream)), "tp_sync")
        self._pending = False

    def close(self) -> None:
        """Unmap the peers and free this rank's buffers (after all GPU work that uses them)."""
        self._views = [None, None]
        for p in self._opened:
            self._lib.fa_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if getattr(self, "_local", 0):
            self._lib.fa_ipc_free(ctypes.c_void_p(self._local))
            self._local = 0
