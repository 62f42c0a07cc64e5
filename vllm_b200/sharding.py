"""Multi-GPU partitioning of the decode path (one process per GPU).

Request sharding: decode rows are independent, so each GPU owns a disjoint set
of requests, its own page pool and block tables, and no data-path collective
is needed.  Rows are assigned longest-first to the GPU with the least attended
tokens so far (greedy LPT), which bounds the slowest GPU to within one row of
the mean.  KV-head sharding splits the 8 KV heads (and their 4 query heads
each) evenly over 1, 2, 4 or 8 GPUs: every GPU keeps all pages and the same
block tables, but only its heads' channels, and the per-rank attention
outputs are all-gathered into the model's [B, 2048] rows.
"""
from __future__ import annotations

import heapq

import numpy as np


def shard_by_request(lens, world: int) -> list[np.ndarray]:
    """Row indices per rank (each sorted ascending), balanced by sum of L."""
    lens = np.asarray(lens, dtype=np.int64)
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(lens.size), key=lambda j: (-int(lens[j]), j)):
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


def shard_by_kv_head(world: int, kv_heads: int = 8) -> list[range]:
    """KV heads per rank: contiguous ranges of kv_heads / world."""
    if world <= 0 or kv_heads % world:
        raise ValueError("world must divide the number of KV heads")
    per = kv_heads // world
    return [range(r * per, (r + 1) * per) for r in range(world)]


def head_channels(heads: range, head_dim: int = 64, group: int = 1) -> slice:
    """Channel slice of ``heads`` in a row of ``group`` x head_dim channels per head
    (group 1: a KV pool row; group 4: a q or attention-output row)."""
    return slice(heads.start * group * head_dim, heads.stop * group * head_dim)


def slice_kv_heads(pool, heads: range):
    """A rank's pool [layers, pages, 16, len(heads) * 64] cut from the model's
    [layers, pages, 16, 8 * 64]: same pages, same block tables, fewer channels."""
    return pool[..., head_channels(heads)]


def slice_q_heads(q, heads: range):
    """A rank's query rows [B, 4 * len(heads) * 64] (query heads 4k .. 4k + 3 of
    each of its KV heads k)."""
    return q[..., head_channels(heads, group=4)]


def interleave_head_shards(gathered):
    """[world, B, 4 * kv_per_rank * 64] -> [B, world * 4 * kv_per_rank * 64]:
    the all-gathered per-rank outputs back in the model's head-major row
    layout (rank r's heads are contiguous and ranks own increasing heads)."""
    world, batch, width = gathered.shape
    if hasattr(gathered, "permute"):
        return gathered.permute(1, 0, 2).reshape(batch, world * width)
    return gathered.transpose(1, 0, 2).reshape(batch, world * width)


def all_gather_head_shards(local, gathered_flat, group=None):
    """All-gathers every rank's [B, width] attention slice over ``group`` into
    the first world * B rows of ``gathered_flat`` ([>= world * B, width]) and
    returns the [B, world * width] model rows."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    batch, width = local.shape
    gathered = gathered_flat[:world * batch]
    dist.all_gather_into_tensor(gathered, local, group=group)
    return interleave_head_shards(gathered.view(world, batch, width))


class HeadShardedDecode:
    """One rank of KV-head-sharded decode attention: rank r holds KV heads
    ``shard_by_kv_head(world)[r]`` of every page and ``attend`` returns the
    model's [B, 2048] attention rows on every rank.

    mode "p2p": the all-gather is fused into the decode kernel
    (``tvp_paged_decode_attention_gather``): each output group is stored
    straight into every rank's gathered rows over NVLink, and the launch ends
    once all ranks' rows have landed (bounded wait in its last CTA).  The rows live in two buffers
    used alternately, so the rows ``attend`` returns stay valid until the call
    after next.  mode "nccl": the decode writes this rank's slice and an NCCL
    all-gather plus an interleave assembles the rows.

    Every rank makes the same calls in the same order.  Buffers are allocated
    once for ``max_batch`` rows.
    """

    def __init__(self, max_batch: int, group=None, device=None, num_ctas: int = 0,
                 mode: str = "p2p"):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _native as N
        from . import ops

        if mode not in ("p2p", "nccl"):
            raise ValueError("mode must be 'p2p' or 'nccl'")
        self.mode = mode
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.heads = shard_by_kv_head(self.world)[self.rank]
        self.kv_heads = len(self.heads)
        self.device = torch.device(device if device is not None else "cuda")
        self.max_batch = max_batch
        self.workspace = ops.DecodeWorkspace(max_batch, self.device, num_ctas=num_ctas,
                                             kv_heads=self.kv_heads)
        self.width = 4 * self.kv_heads * 64
        self._h = None
        if mode == "nccl":
            self.local = torch.empty((max_batch, self.width), dtype=torch.bfloat16,
                                     device=self.device)
            # flat [world * B, width]: rank r's rows at [r B, (r + 1) B) for any B <= max_batch
            self.gathered = torch.empty((self.world * max_batch, self.width),
                                        dtype=torch.bfloat16, device=self.device)
            return
        lib = N.load()
        with torch.cuda.device(self.device):
            # Every fallible local step is followed by an agreement across the
            # group, so that a failure on one rank makes every rank stop at the
            # same point instead of leaving the others waiting in a collective.
            h = ctypes.c_void_p()
            mine = (ctypes.c_char * N.TVP_IPC_HANDLE_BYTES)()
            rc = lib.tvp_head_gather_create(self.world, self.rank, self.kv_heads, max_batch,
                                            ctypes.byref(h))
            if rc == N.TVP_OK:
                self._h = h
                rc = lib.tvp_head_gather_export(h, mine)
            self._agree(rc, "tvp_head_gather_create / export", connected=False)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(mine), group=group)
            rc = lib.tvp_head_gather_connect(h, b"".join(handles))
            self._agree(rc, "tvp_head_gather_connect", connected=True)
            self.rows = []
            for b in (0, 1):
                ptr = ctypes.c_void_p()
                N.check(lib.tvp_head_gather_rows(h, b, ctypes.byref(ptr)), "tvp_head_gather_rows")
                from .cache import _CudaArray
                self.rows.append(torch.as_tensor(
                    _CudaArray(ptr.value, (max_batch, 2048), "<u2"), device=self.device
                ).view(torch.bfloat16))
        self.buffer = 0

    def _agree(self, rc: int, what: str, connected: bool):
        """All ranks learn every rank's status; if any failed, every rank
        tears down its group (IPC-safe order) and raises."""
        from . import _native as N
        statuses = [None] * self.world
        self.dist.all_gather_object(statuses, int(rc), group=self.group)
        if all(st == N.TVP_OK for st in statuses):
            return
        if self._h is not None:
            lib = N.load()
            if connected:
                lib.tvp_head_gather_disconnect(self._h)
            self.dist.barrier(group=self.group)  # no peer maps our buffer any more
            lib.tvp_head_gather_destroy(self._h)
            self._h = None
        else:
            self.dist.barrier(group=self.group)
        bad = {r: st for r, st in enumerate(statuses) if st != N.TVP_OK}
        raise RuntimeError(f"{what} failed on ranks {bad}")

    def plan(self, seq_lens, table_stride: int, error=None, stream=None):
        from . import ops
        ops.decode_plan(seq_lens, table_stride, self.workspace, error=error, stream=stream)

    def attend(self, q_local, k_pool, v_pool, layer, block_tables, seq_lens, error=None,
               gather=True, stream=None, scale=0.125):
        """Decode attention of this rank's heads, then the rows of all heads
        ([B, 2048] on every rank).  ``gather=False`` (nccl mode) returns this
        rank's [B, 4 * kv_heads * 64] slice without the collective."""
        from . import _native as N
        from . import ops
        batch = seq_lens.numel()
        if self.mode == "nccl" or not gather:
            if self.mode != "nccl":
                raise ValueError("gather=False needs mode='nccl'")
            local = self.local[:batch]
            ops.paged_decode_attention(q_local, k_pool, v_pool, layer, block_tables, seq_lens,
                                       self.workspace, out=local, scale=scale, error=error,
                                       stream=stream)
            if not gather:
                return local
            return all_gather_head_shards(local, self.gathered, self.group)
        if self.workspace.batch != batch:
            raise ValueError("plan() this batch first")
        lib = N.load()
        num_layers, num_pages, kv_heads = ops._pool_geometry(k_pool, v_pool)
        if kv_heads != self.kv_heads or q_local.shape != (batch, self.width):
            raise ValueError("pools / q do not hold this rank's heads")
        st = ops._stream(stream)
        rc = lib.tvp_paged_decode_attention_gather(
            ops._ptr(q_local), ops._ptr(k_pool), ops._ptr(v_pool), num_pages, num_layers, layer,
            kv_heads, 4 * kv_heads, ops._ptr(block_tables), block_tables.shape[1],
            ops._ptr(seq_lens), batch, float(scale), self.workspace.num_ctas,
            ops._ptr(self.workspace.buffer), self.workspace.nbytes, self._h, self.buffer,
            ops._ptr(error), st)
        N.check(rc, "tvp_paged_decode_attention_gather")
        rows = self.rows[self.buffer][:batch]
        self.buffer ^= 1
        return rows

    def close(self):
        """Frees the gather buffers; every rank calls it.  Every rank first
        stops writing and closes its peers' buffers, then (after a barrier)
        frees its own, which no peer maps any more."""
        if self._h is None:
            return
        import torch

        from . import _native as N
        lib = N.load()
        torch.cuda.synchronize(self.device)
        self.dist.barrier(group=self.group)
        N.check(lib.tvp_head_gather_disconnect(self._h), "tvp_head_gather_disconnect")
        self.dist.barrier(group=self.group)
        N.check(lib.tvp_head_gather_destroy(self._h), "tvp_head_gather_destroy")
        self._h = None
        self.rows = []


def imbalance(lens, shards) -> float:
    """max over ranks of sum L divided by the mean (1.0 = perfect)."""
    lens = np.asarray(lens, dtype=np.int64)
    loads = [int(lens[s].sum()) for s in shards]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0
