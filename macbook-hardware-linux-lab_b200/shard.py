"""Host logic for running the decode path on several GPUs of one node.

One process per GPU (torch.distributed over NCCL for the plumbing; gloo on
CPU for the tests of this logic).  The reference runs on a single GPU with a
single in-order queue (qwen_server.c:733-738) and has no multi-GPU path; this
module adds the two ways the decode step shards:

* by sequence -- independent sequences are dealt to GPUs, longest first onto
  the least-loaded GPU (balances KV bytes, not counts); no data-path
  collective;
* by KV range -- one long sequence's cache rows are cut into contiguous
  ranges, one per GPU; each GPU produces a partial (m, l, o) per q head over
  its rows and the partials are merged with a log-sum-exp combine -- the
  cross-GPU form of the reference's split-K segment reduce
  (kernel_attention_gqa.cl:378-397).  KvShardExchangeDecoder does the
  exchange and merge in one kernel over peer memory (NVLink stores and
  flags); KvShardDecoder all-gathers the partials with the process group's
  collective (NCCL) and merges them in a second kernel.
"""
from __future__ import annotations

import heapq

HEAD_DIM = 128


def plan_sequence_shards(lengths, world: int) -> list[list[int]]:
    """Sequence indices per rank: LPT (longest first, to the rank with the
    fewest rows so far; ties to the lower rank).  Deterministic."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(s) for s in shards]


def plan_kv_ranges(total_rows: int, world: int, quantum: int = 32) -> list[tuple[int, int]]:
    """(begin, rows) per rank covering [0, total_rows): contiguous, in rank
    order, every range that does not end at total_rows a multiple of
    `quantum` rows, sizes as equal as that allows (trailing ranks may be
    empty for short caches)."""
    if world < 1 or total_rows < 0 or quantum < 1:
        raise ValueError("bad plan arguments")
    units = -(-total_rows // quantum)
    base, extra = divmod(units, world)
    out, begin = [], 0
    for r in range(world):
        n = (base + (1 if r < extra else 0)) * quantum
        n = max(0, min(n, total_rows - begin))
        out.append((begin, n))
        begin += n
    return out


def packed_width(n_rows: int) -> int:
    """Floats of one packed partial: m[n_rows] | l[n_rows] | o[n_rows * 128]."""
    return n_rows * (2 + HEAD_DIM)


def all_gather_partials(packed, group=None):
    """All-gathers one packed partial per rank (a 1-D tensor of
    packed_width floats, on the rank's GPU for NCCL or on the CPU for gloo)
    into a [world, width] tensor in rank order."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return packed.view(1, -1)  # a single process: nothing to exchange
    world = dist.get_world_size(group)
    flat = torch.empty(world * packed.numel(), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(flat, packed.contiguous().view(-1), group=group)
    return flat.view(world, packed.numel())


class KvShardDecoder:
    """One layer's decode on this rank's KV range (rows [begin, begin+rows)
    of a cache of `total_rows`), combined across ranks.  `ctx` is a
    gqa_b200 Context on this rank's GPU; `k_local`/`v_local` are this rank's
    [n_kv][rows_capacity][128] caches."""

    def __init__(self, ctx, k_local, v_local, begin: int, rows: int, group=None):
        import torch
        from .gqa import kv_of
        self.ctx, self.begin, self.rows, self.group = ctx, begin, rows, group
        self.kv = kv_of(k_local, v_local)
        self._keep = (k_local, v_local)
        self.n_q = ctx.n_heads_q
        self.width = packed_width(self.n_q)
        self.part = torch.empty(self.width, device=k_local.device)

    def step(self, qkv, pos: int, out) -> None:
        """qkv: the new token's [q|k|v] row (same on every rank); out: [n_q*128]."""
        base = self.part.data_ptr()
        n = self.n_q
        self.ctx.decode_kv_shard(self.kv, qkv, pos, self.begin, self.rows, base, base + 4 * n,
                                 base + 8 * n)
        gathered = all_gather_partials(self.part, self.group)
        self.ctx.lse_combine_packed(gathered.shape[0], n, gathered, self.width, out)


class KvShardExchangeDecoder:
    """KvShardDecoder with the exchange done by the merging kernel itself:
    each rank stores its merged partial into every rank's inbox over NVLink
    and merges the world partials once their flags are up
    (gqa_decode_kv_shard_exchange).  The process group is used once, to swap
    the inbox handles; the data path uses no collective."""

    def __init__(self, ctx, k_local, v_local, begin: int, rows: int, group=None):
        import torch.distributed as dist
        from .gqa import Exchange, kv_of
        if dist.is_available() and dist.is_initialized():
            rank, world = dist.get_rank(group), dist.get_world_size(group)
        else:
            rank, world = 0, 1
        self.ctx, self.begin, self.rows = ctx, begin, rows
        self.kv = kv_of(k_local, v_local)
        self._keep = (k_local, v_local)
        self.exchange = Exchange(ctx, rank, world)
        handles = [self.exchange.handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, self.exchange.handle, group=group)
        self.exchange.open(handles)

    def step(self, qkv, pos: int, out, stream=None) -> None:
        """qkv: the new token's [q|k|v] row (same on every rank); out: [n_q*128]."""
        self.exchange.step(self.kv, qkv, pos, self.begin, self.rows, out, stream)

    def close(self) -> None:
        self.exchange.destroy()
