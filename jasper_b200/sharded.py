"""Range-sharded index across the ranks of a torch.distributed group.

One process per GPU.  Rank r owns the global ids [offset_r, offset_r + n_r)
of an index of n_total rows (``shard_range``) and builds its own sub-graph
over them; neighbour ids are stored global and the entry point is the
shard's first row (``jb_graph_apply_global_offset``, the reference's
graph::apply_global_offset, include/jasper/index/graph.cuh:801-827).  A
query batch is searched by every rank on its own shard; each rank's top-k
(global ids) is gathered to the root over NCCL and merged there by
``jb_merge_topk`` (ties by id).  The reference has no multi-GPU path; this is
the range-sharded mode the port adds for indexes larger than one GPU.

Small indexes are better served by replicas with the queries split across
ranks (no exchange at all); ``split_queries`` gives each rank its slice.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import Graph, _lib

__all__ = ["shard_range", "split_queries", "gather_topk", "merge_topk", "ShardedGraph"]


def shard_range(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(offset, count) of rank's contiguous id range; the first n_total % world
    ranks hold one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_total, world)
    count = base + (1 if rank < extra else 0)
    offset = rank * base + min(rank, extra)
    return offset, count


def split_queries(n_queries: int, world: int, rank: int) -> slice:
    """The contiguous slice of a query batch a replica searches."""
    off, cnt = shard_range(n_queries, world, rank)
    return slice(off, off + cnt)


def gather_topk(local_idx: torch.Tensor, local_dist: torch.Tensor, root: int = 0,
                group=None, out: torch.Tensor | None = None
                ) -> tuple[torch.Tensor, torch.Tensor] | None:
    """Collect every rank's [nq, k] top-k on ``root`` with ONE collective.
    Each rank packs its ids and distance bits into one [2, nq, k] int32
    slice of a [world, 2, nq, k] buffer (``out`` if given: reused across
    calls) and the slices are exchanged with all_gather_into_tensor (one
    NCCL all-gather: each shard's 8 nq k bytes reach every rank; the
    lowest host cost of the collectives that gather).  Returns ``(ids,
    dists)`` as [world, nq, k] views of the buffer on ``root`` (shard stride
    2 nq k, which ``merge_topk`` reads in place) and None elsewhere."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nq, k = local_idx.shape
    if out is None or out.shape != (world, 2, nq, k) or out.device != local_idx.device:
        out = torch.empty(world, 2, nq, k, dtype=torch.int32, device=local_idx.device)
    mine = out[rank]
    mine[0].copy_(local_idx)
    mine[1].copy_(local_dist.to(torch.float32).view(torch.int32))
    dist.all_gather_into_tensor(out.view(-1), mine.reshape(-1), group=group)
    if rank != root:
        return None
    return out[:, 0], out[:, 1].view(torch.float32)


def merge_topk(shard_idx: torch.Tensor, shard_dist: torch.Tensor,
               k: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge [n_shards, nq, k] per-shard top-k lists (CUDA tensors) into the
    global [nq, k] by (distance, id) with jb_merge_topk_strided.  The shard
    dimension may have any stride >= nq * k (the views ``gather_topk``
    returns are read in place); the inner [nq, k] must be contiguous."""
    if not shard_idx.is_cuda or not shard_dist.is_cuda:
        raise ValueError("merge_topk needs CUDA tensors")
    ns, nq, kk = shard_idx.shape
    k = kk if k is None else k
    if k != kk:
        raise ValueError("k must equal the per-shard k")

    def prep(t, dtype):
        if t.dtype != dtype or t.stride(1) != kk or t.stride(2) != 1 or t.stride(0) < nq * kk:
            t = t.to(dtype).contiguous()
        return t
    si = prep(shard_idx, torch.int32)
    sd = prep(shard_dist, torch.float32)
    if si.stride(0) != sd.stride(0):
        si, sd = si.contiguous(), sd.contiguous()
    oi = torch.empty(nq, k, dtype=torch.int32, device=si.device)
    od = torch.empty(nq, k, dtype=torch.float32, device=si.device)
    _lib.call("jb_merge_topk_strided", si.data_ptr(), sd.data_ptr(), si.stride(0), ns, nq, k,
              oi.data_ptr(), od.data_ptr(), torch.cuda.current_stream(si.device).cuda_stream)
    return oi, od


class ShardedGraph:
    """This rank's shard of a range-sharded index."""

    def __init__(self, graph: Graph, offset: int, n_total: int, group=None):
        self.graph = graph
        self.offset = offset
        self.n_total = n_total
        self.group = group
        self._gather_buf = None   # root's [world, 2, nq, k] gather buffer, reused

    @classmethod
    def build(cls, local_vectors: torch.Tensor, offset: int, n_total: int, group=None,
              **build_kwargs) -> "ShardedGraph":
        """Build this rank's sub-graph over its rows (global ids offset + i)."""
        g = Graph.build(local_vectors, **build_kwargs)
        if offset:
            _lib.call("jb_graph_apply_global_offset", g._handle, C.c_uint32(offset))
        return cls(g, offset, n_total, group)

    def search_local(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64):
        """This shard's top-k (global ids) for all queries."""
        return self.graph.search(queries, k=k, beam_width=beam_width)

    def search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64, root: int = 0,
               phases: list | None = None):
        """All ranks call this with the same queries.  Returns the merged
        global top-k on ``root`` and None elsewhere.  With ``phases`` (a
        list), appends CUDA events (start, searched, gathered, merged) on the
        current stream, for per-phase timing."""
        ev = None
        if phases is not None:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record()
        li, ld = self.search_local(queries, k, beam_width)
        if ev is not None:
            ev[1].record()
        if self._gather_buf is None or self._gather_buf.shape[2:] != li.shape:
            import torch.distributed as dist
            self._gather_buf = torch.empty(dist.get_world_size(self.group), 2, *li.shape,
                                           dtype=torch.int32, device=li.device)
        g = gather_topk(li, ld, root=root, group=self.group, out=self._gather_buf)
        if ev is not None:
            ev[2].record()
        out = None if g is None else merge_topk(g[0], g[1], k)
        if ev is not None:
            ev[3].record()
            phases.append(ev)
        return out

    def search_host(self, queries: torch.Tensor, out_idx: torch.Tensor, out_dist: torch.Tensor,
                    k: int = 10, beam_width: int = 64, root: int = 0) -> bool:
        """search() from host buffers: ``queries`` [nq, dim] fp16 and, on
        ``root``, ``out_idx`` / ``out_dist`` [nq, k] on the host (page-locked
        for speed).  With one shard the C ABI's host-buffer search runs (the
        kernel reads page-locked queries and writes the results in place);
        with several, the queries are uploaded asynchronously, searched,
        exchanged and merged, and the merged top-k is copied into the output
        buffers.  Synchronous; returns True on ``root``."""
        import torch.distributed as dist
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if queries.is_cuda or out_idx.is_cuda or out_dist.is_cuda:
            raise ValueError("search_host takes host tensors")
        q = queries.contiguous()
        if world == 1:
            if not (out_idx.is_contiguous() and out_dist.is_contiguous()):
                raise ValueError("output buffers must be contiguous")
            limit = beam_width * 2
            _lib.call("jb_graph_search_host", self.graph._handle, q.data_ptr(), q.shape[0],
                      q.shape[1], out_idx.data_ptr(), out_dist.data_ptr(), k, beam_width, limit,
                      torch.cuda.current_stream().cuda_stream)
            return True
        dev = torch.device("cuda", torch.cuda.current_device())
        res = self.search(q.to(dev, non_blocking=True), k=k, beam_width=beam_width, root=root)
        if res is not None:
            out_idx.copy_(res[0], non_blocking=True)
            out_dist.copy_(res[1], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return res is not None

    def free(self):
        self.graph.free()
