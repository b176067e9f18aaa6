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
                group=None) -> tuple[torch.Tensor, torch.Tensor] | None:
    """Gather every rank's [nq, k] top-k to ``root`` as [n_shards, nq, k]
    tensors (rank order); other ranks get None."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    li = local_idx.contiguous()
    ld = local_dist.contiguous()
    if rank == root:
        gi = [torch.empty_like(li) for _ in range(world)]
        gd = [torch.empty_like(ld) for _ in range(world)]
        dist.gather(li, gi, dst=root, group=group)
        dist.gather(ld, gd, dst=root, group=group)
        return torch.stack(gi), torch.stack(gd)
    dist.gather(li, None, dst=root, group=group)
    dist.gather(ld, None, dst=root, group=group)
    return None


def merge_topk(shard_idx: torch.Tensor, shard_dist: torch.Tensor,
               k: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge [n_shards, nq, k] per-shard top-k lists (CUDA tensors) into the
    global [nq, k] by (distance, id) with jb_merge_topk."""
    if not shard_idx.is_cuda or not shard_dist.is_cuda:
        raise ValueError("merge_topk needs CUDA tensors")
    ns, nq, kk = shard_idx.shape
    k = kk if k is None else k
    si = shard_idx.to(torch.int32).contiguous()
    sd = shard_dist.to(torch.float32).contiguous()
    oi = torch.empty(nq, k, dtype=torch.int32, device=si.device)
    od = torch.empty(nq, k, dtype=torch.float32, device=si.device)
    if k != kk:
        raise ValueError("k must equal the per-shard k")
    _lib.call("jb_merge_topk", si.data_ptr(), sd.data_ptr(), ns, nq, k, oi.data_ptr(),
              od.data_ptr(), torch.cuda.current_stream(si.device).cuda_stream)
    return oi, od


class ShardedGraph:
    """This rank's shard of a range-sharded index."""

    def __init__(self, graph: Graph, offset: int, n_total: int, group=None):
        self.graph = graph
        self.offset = offset
        self.n_total = n_total
        self.group = group

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

    def search(self, queries: torch.Tensor, k: int = 10, beam_width: int = 64, root: int = 0):
        """All ranks call this with the same queries.  Returns the merged
        global top-k on ``root`` and None elsewhere."""
        li, ld = self.search_local(queries, k, beam_width)
        g = gather_topk(li, ld, root=root, group=self.group)
        if g is None:
            return None
        return merge_topk(g[0], g[1], k)

    def free(self):
        self.graph.free()
