"""Host-side mirror of the reference's paged KV interface over the HBM pool.

Same names, argument meaning and error behaviour as lltsdyp/flour:

* ``BlockAllocator``  src/models/common/paged.rs:7-53   (refcounted free list, host only)
* ``BlockTable``      src/models/common/paged.rs:57-122 (logical -> physical, ``slot``/``slots``)
* ``PagedKvPool``     src/models/common/paged.rs:129-280 (now device slabs
  [num_blocks, kv_heads, block_size, head_dim] per layer; ``write`` is reshape_and_cache,
  ``write_block`` is fa_write_block, ``block_view`` is a zero-copy view)
* ``KvCache``         src/models/common/cache.rs:12-97, 429-458 (one sequence's allocator, table
  and pool; ``allocate_kv`` / ``write_kv`` / ``kv_blocks``)
* ``paged_attention`` src/backend/cpu.rs:57-112 — q (b, Hq, seq_q, d), the blocks of a sequence,
  n_rep, scale -> (b, Hq, seq_q, d) in q's dtype, computed by the CUDA kernels.

Reference errors (``candle_core::bail!``) become ``ValueError`` here; C-ABI failures raise
``FlourAttnError``. ``build_batch`` (new) turns many sequences' tables into the int32 block
tables / context lengths / slot mapping the batched kernels take.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


class BlockAllocator:
    """paged.rs:7-53. The first ``allocate`` returns block 0."""

    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks - 1, -1, -1))
        self.ref_counts = [0] * num_blocks

    def allocate(self):
        if not self.free:
            return None
        i = self.free.pop()
        self.ref_counts[i] = 1
        return i

    def incref(self, block_id: int) -> None:
        self.ref_counts[block_id] += 1

    def decref(self, block_id: int) -> bool:
        assert self.ref_counts[block_id] > 0, "decref of unreferenced block"
        self.ref_counts[block_id] -= 1
        if self.ref_counts[block_id] == 0:
            self.free.append(block_id)
            return True
        return False

    def ref_count(self, block_id: int) -> int:
        return self.ref_counts[block_id]

    def num_free(self) -> int:
        return len(self.free)


class BlockTable:
    """paged.rs:57-122."""

    def __init__(self, block_size: int):
        self._blocks: list[int] = []
        self._block_size = block_size
        self._len = 0

    def len(self) -> int:
        return self._len

    def is_empty(self) -> bool:
        return self._len == 0

    def block_size(self) -> int:
        return self._block_size

    def capacity(self) -> int:
        return len(self._blocks) * self._block_size

    def push_block(self, block_id: int) -> None:
        self._blocks.append(block_id)

    def blocks(self) -> list[int]:
        return list(self._blocks)

    def block_at(self, logical_block: int) -> int:
        return self._blocks[logical_block]

    def clear(self) -> None:
        self._blocks.clear()
        self._len = 0

    def advance(self, n: int) -> None:
        self._len += n

    def slot(self, pos: int) -> int:
        # Positions are unsigned in the reference (paged.rs:114-116 indexes with a usize): a
        # negative one is out of range like one past the last block, not the last block's slot.
        if pos < 0:
            raise IndexError(f"slot position {pos} out of range")
        return self._blocks[pos // self._block_size] * self._block_size + pos % self._block_size

    def slots(self, start: int, end: int) -> list[int]:
        return [self.slot(p) for p in range(start, end)]


class PagedKvPool:
    """paged.rs:129-280 with the slabs in HBM, layout [num_blocks, kv_heads, block_size, d]."""

    def __init__(self, num_layers: int, num_blocks: int, kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device, block_size: int = 16):
        self.block_size = block_size
        self._kv_heads = kv_heads
        self._head_dim = head_dim
        shape = (num_blocks, kv_heads, block_size, head_dim)
        self.k_pools = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v_pools = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]

    def num_layers(self) -> int:
        return len(self.k_pools)

    def num_blocks(self) -> int:
        return self.k_pools[0].shape[0]

    def kv_heads(self) -> int:
        return self._kv_heads

    def head_dim(self) -> int:
        return self._head_dim

    def dtype(self) -> torch.dtype:
        return self.k_pools[0].dtype

    def write(self, layer_idx: int, slots, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: (1, kv_heads, n, d) as the reference passes them; one reshape_and_cache launch
        scatters token i to slots[i] (paged.rs:186-204)."""
        kt, vt = k.squeeze(0), v.squeeze(0)  # (kv_heads, n, d)
        sm = torch.as_tensor(list(slots) if not torch.is_tensor(slots) else slots,
                             dtype=torch.int32).to(kt.device)
        ops.reshape_and_cache(self.k_pools[layer_idx], self.v_pools[layer_idx],
                              kt.transpose(0, 1), vt.transpose(0, 1), sm)

    @staticmethod
    def _normalize_block(t: torch.Tensor) -> torch.Tensor:
        # paged.rs:244-250
        if t.dim() == 4:
            if t.shape[0] != 1:
                raise ValueError(f"cannot squeeze dim 0 of size {t.shape[0]}")
            return t.squeeze(0)
        if t.dim() == 3:
            return t
        raise ValueError(f"write_block expects rank 3 or 4 tensor, got rank {t.dim()}")

    def write_block(self, layer_idx: int, block_id: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """paged.rs:211-240: overwrite one full physical block; the same shape checks."""
        kt, vt = self._normalize_block(k), self._normalize_block(v)
        if tuple(kt.shape) != tuple(vt.shape):
            raise ValueError(f"write_block k/v shape mismatch: k={tuple(kt.shape)} v={tuple(vt.shape)}")
        kh, bs, hd = kt.shape
        if kh != self._kv_heads or hd != self._head_dim:
            raise ValueError(
                f"write_block expects (.., kv_heads={self._kv_heads}, block_size, head_dim="
                f"{self._head_dim}), got kv_heads={kh} head_dim={hd}")
        if bs != self.block_size:
            raise ValueError(f"write_block expects block_size {self.block_size}, got {bs}")
        ops.write_block(self.k_pools[layer_idx], self.v_pools[layer_idx], block_id,
                        kt.to(self.dtype()), vt.to(self.dtype()))

    def block_view(self, layer_idx: int, start_slot: int, n: int):
        """paged.rs:266-279: zero-copy (1, kv_heads, n, d) views of n slots inside one block."""
        blk, off = divmod(start_slot, self.block_size)
        if off + n > self.block_size:
            raise ValueError("block_view spans more than one physical block")
        k = self.k_pools[layer_idx][blk, :, off:off + n, :].unsqueeze(0)
        v = self.v_pools[layer_idx][blk, :, off:off + n, :].unsqueeze(0)
        return k, v

    def gather(self, layer_idx: int, slots):
        """paged.rs:255-260: read an arbitrary slot list as (1, kv_heads, n, d)."""
        s = torch.as_tensor(list(slots), dtype=torch.long, device=self.k_pools[0].device)
        blk, off = s // self.block_size, s % self.block_size
        k = self.k_pools[layer_idx][blk, :, off, :].transpose(0, 1).unsqueeze(0)
        v = self.v_pools[layer_idx][blk, :, off, :].transpose(0, 1).unsqueeze(0)
        return k, v


@dataclass
class SequenceBlocks:
    """What ``KvCache.kv_blocks`` hands to ``paged_attention``: the layer's slabs plus this
    sequence's logical->physical block list and live length (the reference returns one view
    per logical block, cache.rs:83-96; the kernels walk the same blocks through the table)."""

    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_table: list[int]
    kv_len: int


class KvCache:
    """cache.rs:12-97 + Cache::allocate_kv/write_kv/kv_blocks (cache.rs:429-458), one sequence."""

    def __init__(self, num_layers: int, max_seq_len: int, kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device, block_size: int = 16):
        num_blocks = -(-max_seq_len // block_size)
        self.max_seq_len = max_seq_len
        self.pool = PagedKvPool(num_layers, num_blocks, kv_heads, head_dim, dtype, device,
                                block_size)
        self.allocator = BlockAllocator(num_blocks)
        self.table = BlockTable(block_size)

    def allocate(self):
        b = self.allocator.allocate()
        if b is not None:
            self.table.push_block(b)
        return b

    def len(self) -> int:
        return self.table.len()

    def capacity(self) -> int:
        return self.table.capacity()

    def slots(self, start: int, end: int) -> list[int]:
        return self.table.slots(start, end)

    def advance(self, n: int) -> None:
        self.table.advance(n)

    def allocate_kv(self, seq_len: int) -> None:
        start = self.table.len()
        end = start + seq_len
        if end > self.max_seq_len:
            raise ValueError(
                f"paged kv cache overflow: {end} tokens exceeds max_seq_len {self.max_seq_len}")
        while self.table.capacity() < end:
            if self.allocate() is None:
                raise ValueError("out of kv blocks")
        self.table.advance(seq_len)

    def write_kv(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """write_current (cache.rs:71-77): the trailing seq_len tokens go to their slots."""
        seq_len = k.shape[2]
        end = self.table.len()
        self.pool.write(layer_idx, self.table.slots(end - seq_len, end), k, v)

    def kv_blocks(self, layer_idx: int) -> SequenceBlocks:
        n = -(-self.table.len() // self.table.block_size())
        return SequenceBlocks(self.pool.k_pools[layer_idx], self.pool.v_pools[layer_idx],
                              self.table.blocks()[:n], self.table.len())

    def reset_sequence(self) -> None:
        for b in self.table.blocks():
            self.allocator.decref(b)
        self.table.clear()


def paged_attention(q: torch.Tensor, blocks: SequenceBlocks, n_rep: int, scale: float,
                    workspace: ops.Workspace | None = None) -> torch.Tensor:
    """cpu.rs:57-112 on the GPU: q (b, Hq, seq_q, d) -> (b, Hq, seq_q, d) in q.dtype.

    Every batch row attends to the same block list (the reference's b is always 1)."""
    b, hq, sq, d = q.shape
    kv_len = blocks.kv_len
    if kv_len < sq:
        raise ValueError(f"kv_len {kv_len} shorter than seq_q {sq}")
    dev = q.device
    nblk = max(len(blocks.block_table), 1)
    table = torch.tensor([blocks.block_table] * b, dtype=torch.int32, device=dev).reshape(b, nblk) \
        if blocks.block_table else torch.zeros((b, 1), dtype=torch.int32, device=dev)
    qp = q.permute(0, 2, 1, 3).reshape(b * sq, hq, d).contiguous()
    cu = torch.arange(0, (b + 1) * sq, sq, dtype=torch.int32, device=dev)
    ctx = torch.full((b,), kv_len, dtype=torch.int32, device=dev)
    if workspace is None:
        workspace = ops.Workspace(dev)
    out = ops.paged_attention_varlen(qp, blocks.k_cache, blocks.v_cache, cu, ctx, table, n_rep,
                                     scale, sq, kv_len, workspace)
    return out.reshape(b, sq, hq, d).permute(0, 2, 1, 3).contiguous()


@dataclass
class BatchMetadata:
    block_tables: torch.Tensor   # int32 [B, max_blocks]
    context_lens: torch.Tensor   # int32 [B]
    cu_seqlens_q: torch.Tensor   # int32 [B+1]
    slot_mapping: torch.Tensor   # int32 [sum q_len]
    max_context_len: int
    max_seqlen_q: int


def build_batch(tables: list[BlockTable], q_lens: list[int], device) -> BatchMetadata:
    """Batched form of the per-sequence bookkeeping (cache.rs:71-96): one int32 block-table
    row per sequence, its live length, and the slots of its trailing q_len new tokens. Raises the
    C++ host's errors for lists of different lengths and for a q_len outside [0, len]."""
    if len(tables) != len(q_lens):
        raise ValueError("build_batch: tables and q_lens differ in length")
    for t, n in zip(tables, q_lens):
        if n < 0 or n > t.len():
            raise ValueError("build_batch: q_len exceeds the sequence length")
    B = len(tables)
    max_blocks = max(1, max(len(t.blocks()) for t in tables)) if tables else 1
    bt = torch.zeros((B, max_blocks), dtype=torch.int32)
    ctx = torch.zeros(B, dtype=torch.int32)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    slots: list[int] = []
    for i, (t, n) in enumerate(zip(tables, q_lens)):
        blk = t.blocks()
        if blk:
            bt[i, :len(blk)] = torch.tensor(blk, dtype=torch.int32)
        ctx[i] = t.len()
        cu[i + 1] = cu[i] + n
        slots.extend(t.slots(t.len() - n, t.len()))
    return BatchMetadata(bt.to(device), ctx.to(device), cu.to(device),
                         torch.tensor(slots, dtype=torch.int32).to(device),
                         int(ctx.max()) if B else 0, max(q_lens) if q_lens else 0)


def rope_tables(head_dim: int, max_position: int, rope_theta: float, dtype: torch.dtype,
                device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """The RoPE tables of Cache::new (cache.rs:378-392), as the f32 tensors the fused QKV
    kernel reads: theta_i = 1 / rope_theta^(2i / head_dim) and angle = position * theta_i in
    f32, then cos/sin rounded to the model dtype exactly as the reference stores them.

    Host-side setup done once per model; returns (cos, sin), each [max_position, head_dim/2]."""
    half = head_dim // 2
    i = torch.arange(half, dtype=torch.float32)
    theta = 1.0 / torch.pow(torch.tensor(rope_theta, dtype=torch.float32), (2 * i) / head_dim)
    pos = torch.arange(max_position, dtype=torch.float32).reshape(-1, 1)
    ang = pos * theta.reshape(1, half)
    cos = ang.cos().to(dtype).to(torch.float32).contiguous()
    sin = ang.sin().to(dtype).to(torch.float32).contiguous()
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin
