"""Range-sharded index: id ranges, the gather to the root over a process
group (world size 2, gloo on CPU), and the device k-way merge (GPU)."""
import os
import socket

import numpy as np
import pytest
import torch

from jasper_b200 import sharded, synthetic


def test_shard_range_partitions_ids():
    for n in (0, 1, 7, 100, 12_500_001):
        for world in (1, 2, 3, 8):
            parts = [sharded.shard_range(n, world, r) for r in range(world)]
            assert sum(c for _, c in parts) == n
            off = 0
            for o, c in parts:
                assert o == off
                off += c
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    with pytest.raises(ValueError):
        sharded.shard_range(10, 2, 2)
    assert sharded.split_queries(10, 3, 1) == slice(4, 7)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reference_merge(idx: np.ndarray, dist: np.ndarray, k: int):
    """(distance, id) order over all shards; empty slots (-1) last."""
    ns, nq, kk = idx.shape
    out_i = np.full((nq, k), -1, np.int32)
    out_d = np.full((nq, k), 1e30, np.float32)
    for q in range(nq):
        c = [(float(dist[s, q, j]), int(idx[s, q, j])) for s in range(ns) for j in range(kk)
             if idx[s, q, j] >= 0]
        c.sort()
        for j, (d, i) in enumerate(c[:k]):
            out_i[q, j], out_d[q, j] = i, d
    return out_i, out_d


def _gather_worker(rank, world, port, result_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n_total, nq, k = 1000, 6, 5
        off, cnt = sharded.shard_range(n_total, world, rank)
        rng = np.random.default_rng(rank)
        # this rank's top-k: global ids inside its range, sorted distances
        ids = rng.integers(off, off + cnt, size=(nq, k)).astype(np.int32)
        d = np.sort(rng.random((nq, k)).astype(np.float32), axis=1)
        if rank == 1:
            ids[0, 3:] = -1            # a shard with fewer than k results
            d[0, 3:] = 1e30
        got = sharded.gather_topk(torch.from_numpy(ids), torch.from_numpy(d), root=0)
        if rank == 0:
            gi, gd = got
            np.savez(result_path, gi=gi.numpy(), gd=gd.numpy())
        else:
            assert got is None
    finally:
        dist.destroy_process_group()


def test_gather_topk_two_ranks_gloo(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "gathered.npz")
    mp.spawn(_gather_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    z = np.load(out)
    gi, gd = z["gi"], z["gd"]
    assert gi.shape == (2, 6, 5) and gd.shape == (2, 6, 5)
    for r in range(2):
        off, cnt = sharded.shard_range(1000, 2, r)
        rng = np.random.default_rng(r)
        ids = rng.integers(off, off + cnt, size=(6, 5)).astype(np.int32)
        d = np.sort(rng.random((6, 5)).astype(np.float32), axis=1)
        if r == 1:
            ids[0, 3:] = -1
            d[0, 3:] = 1e30
        np.testing.assert_array_equal(gi[r], ids)
        np.testing.assert_array_equal(gd[r], d)
    mi, md = _reference_merge(gi, gd, 5)
    assert (mi[0] >= 0).all()   # the short shard is filled from the other


@pytest.mark.gpu
def test_merge_topk_device_matches_reference(cuda):
    rng = np.random.default_rng(3)
    ns, nq, k = 5, 300, 10
    idx = rng.permutation(ns * nq * k * 3)[:ns * nq * k].reshape(ns, nq, k).astype(np.int32)
    # integer-valued distances: many exact ties, ordered by id
    d = np.sort(rng.integers(0, 20, size=(ns, nq, k)).astype(np.float32), axis=2)
    idx[1, :50, 6:] = -1
    d[1, :50, 6:] = 1e30
    oi, od = sharded.merge_topk(torch.from_numpy(idx).cuda(), torch.from_numpy(d).cuda())
    ri, rd = _reference_merge(idx, d, k)
    np.testing.assert_array_equal(oi.cpu().numpy(), ri)
    np.testing.assert_array_equal(od.cpu().numpy(), rd)


@pytest.mark.gpu
def test_range_sharded_search_single_gpu(cuda):
    """Three shards built and searched on one GPU, merged on the device, equal
    the reference merge of the per-shard results; recall near the unsharded
    graph's at the same beam width."""
    import jasper_b200 as jasper
    from oracle import oracle as O
    n, dim, k, bw = 6000, 96, 10, 32
    X = synthetic.gaussian(n, dim, 91)
    Q = synthetic.gaussian(200, dim, 92)
    q = torch.from_numpy(Q).cuda()
    shards, li, ld = [], [], []
    try:
        for r in range(3):
            off, cnt = sharded.shard_range(n, 3, r)
            sg = sharded.ShardedGraph.build(torch.from_numpy(X[off:off + cnt]).cuda(), off, n,
                                            n_neighbors=32)
            shards.append(sg)
            i, d = sg.search_local(q, k=k, beam_width=bw)
            assert ((i >= off) & (i < off + cnt)).all()
            li.append(i)
            ld.append(d)
        si, sd = torch.stack(li), torch.stack(ld)
        oi, od = sharded.merge_topk(si, sd)
        ri, rd = _reference_merge(si.cpu().numpy(), sd.cpu().numpy(), k)
        np.testing.assert_array_equal(oi.cpu().numpy(), ri)
        np.testing.assert_array_equal(od.cpu().numpy(), rd)
        gt, _ = O.bruteforce(X, Q, k, 0)
        rec = np.mean([len(set(a) & set(b)) / k for a, b in zip(oi.cpu().numpy(), gt)])
        full = jasper.Graph.build(torch.from_numpy(X).cuda(), n_neighbors=32)
        fi, _ = full.search(q, k=k, beam_width=bw)
        rec_full = np.mean([len(set(a) & set(b)) / k for a, b in zip(fi.cpu().numpy(), gt)])
        full.free()
        assert rec >= rec_full - 0.02, (rec, rec_full)
    finally:
        for sg in shards:
            sg.free()
