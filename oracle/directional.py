"""Directional artifacts (cross-polytope LSH, PQ, exact norms) as plain numpy.

TEST INFRASTRUCTURE ONLY (the checker; the product builds these on the GPU).
Restates the reference's artifact builders deterministically:

* LSH edge sketch -- populate_lsh (include/jasper/lsh/lsh_kernels.cuh:9-131):
  Δ = v − u in fp16; sort keys (|Δ| half bits << (B+1)) | sign << B | coord,
  B = 7 (dim ≤ 128, uint8 words) or 15 (uint16 words); k_ranks rounds of
  argmax, each winner stored as its low B+1 bits and then zeroed; edge
  magnitude² = bf16(Σ float(Δ)²).  Only slots below the edge count are
  filled (the reference walks all R slots and reads the rows behind the
  unset ones).
* LSH globals -- accumulate_rank_sums / finalize_lsh_globals
  (lsh_globals.cuh:17-177): c_r = mean over sampled edges of
  |Δ|_(r) / ‖Δ‖, norm_denom = Σ c_r².  Edges are sampled with numpy here
  (the reference uses cuRAND Philox and float atomics, so its values are not
  reproducible anyway).
* PQ -- pq_sample_residuals / pq_kmeans_* / pq_populate
  (pq/pq_kernels.cuh:64-295): Lloyd k-means per subspace on edge residuals,
  codes = argmin with ties to the lower index; norms = Σ x² per row.
* File -- the reference's directional trailer (graph.cuh:1814-1937), written
  after a legacy-layout base section so the reference's loader (which
  computes the trailer offset with the legacy record size, graph.cuh:
  1961-1964) finds it.
"""
from __future__ import annotations

import struct

import numpy as np


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    return ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)


def lsh_edges(X: np.ndarray, edges: np.ndarray, counts: np.ndarray, k_ranks: int):
    """Per-edge packed words [n, R * k_ranks] and bf16 magnitude² [n, R]."""
    n, dim = X.shape
    dpad = (dim + 7) // 8 * 8
    R = edges.shape[1]
    coord_bits = 7 if dpad <= 128 else 15
    wdtype = np.uint8 if coord_bits == 7 else np.uint16
    Xp = np.zeros((n, dpad), np.float16)
    Xp[:, :dim] = X
    packed = np.zeros((n, R * k_ranks), wdtype)
    mag = np.zeros((n, R), np.uint16)
    for u in range(n):
        c = int(counts[u])
        if c == 0:
            continue
        nb = edges[u, :c].astype(np.int64)
        d = (Xp[nb] - Xp[u][None, :]).astype(np.float16)          # fp16 subtraction
        bits = d.view(np.uint16).astype(np.uint32)
        key = ((bits & 0x7FFF) << (coord_bits + 1)) | (((bits >> 15) & 1) << coord_bits) \
            | (np.arange(dpad, dtype=np.uint32)[None, :] & ((1 << coord_bits) - 1))
        f = d.astype(np.float32)
        mag[u, :c] = _bf16_bits((f * f).sum(1, dtype=np.float32))
        order = np.argsort(-key.astype(np.int64), axis=1, kind="stable")[:, :k_ranks]
        win = np.take_along_axis(key, order, axis=1)
        low = (win & ((1 << (coord_bits + 1)) - 1)).astype(wdtype)
        packed[u, :c * k_ranks] = low.reshape(-1)
    return packed, mag


def lsh_globals(X, edges, counts, k_ranks, n_samples=32768, seed=42):
    n, dim = X.shape
    rng = np.random.default_rng(seed)
    qs = rng.integers(0, n, n_samples)
    sums = np.zeros(k_ranks, np.float64)
    nv = 0
    for q in qs:
        c = int(counts[q])
        if c == 0:
            continue
        v = int(edges[q, rng.integers(0, c)])
        d = (X[v].astype(np.float16) - X[q].astype(np.float16)).astype(np.float32)
        nrm = float(np.sqrt((d * d).sum()))
        if nrm == 0.0:
            continue
        mags = np.sort(np.abs(d))[::-1][:k_ranks]
        sums[:len(mags)] += mags / nrm
        nv += 1
    c = (sums / max(nv, 1)).astype(np.float32)
    return c, np.float32((c.astype(np.float32) ** 2).sum(dtype=np.float32))


def pq_train(X, edges, counts, M, n_train=40000, iters=12, seed=123, K=256):
    n, dim = X.shape
    dpad = (dim + 7) // 8 * 8
    assert dpad % M == 0
    dsub = dpad // M
    rng = np.random.default_rng(seed)
    Xp = np.zeros((n, dpad), np.float32)
    Xp[:, :dim] = X.astype(np.float32)
    res = []
    while len(res) < n_train:
        q = int(rng.integers(0, n))
        c = int(counts[q])
        if c == 0:
            continue
        v = int(edges[q, rng.integers(0, c)])
        res.append((X[v].astype(np.float16) - X[q].astype(np.float16)).astype(np.float32))
    T = np.zeros((n_train, dpad), np.float32)
    T[:, :dim] = np.stack(res)
    cent = np.zeros((M, K, dsub), np.float32)
    for j in range(M):
        sub = T[:, j * dsub:(j + 1) * dsub]
        C = sub[rng.choice(n_train, K, replace=False)].copy()
        for _ in range(iters):
            d = ((sub[:, None, :] - C[None]) ** 2).sum(-1)
            lab = d.argmin(1)
            for k in range(K):
                m = lab == k
                if m.any():
                    C[k] = sub[m].mean(0)
        cent[j] = C
    return cent


def pq_codes(X, edges, counts, cent):
    n, dim = X.shape
    M, K, dsub = cent.shape
    R = edges.shape[1]
    dpad = M * dsub
    Xp = np.zeros((n, dpad), np.float16)
    Xp[:, :dim] = X
    codes = np.zeros((n, M * R), np.uint8)
    for u in range(n):
        c = int(counts[u])
        if c == 0:
            continue
        r = (Xp[edges[u, :c]] - Xp[u][None]).astype(np.float16).astype(np.float32)
        for j in range(M):
            d = ((r[:, None, j * dsub:(j + 1) * dsub] - cent[j][None]) ** 2).sum(-1)
            codes[u, j * R:j * R + c] = d.argmin(1)   # subspace-major: code[j * R + e]
    return codes


def norms(X):
    x = X.astype(np.float32)
    return (x * x).sum(1, dtype=np.float32)


def write_legacy_directional(path, X, edges, edist, counts, medoid, R, k_ranks, packed=None,
                             mag=None, c=None, norm_denom=None, cent=None, codes=None, nrm=None):
    """Legacy base records ([vec | count | ids | bf16 dists]) + directional trailer."""
    n, dim = X.shape
    bpn = 2 * dim + 1 + 6 * R
    out = bytearray(struct.pack("<4Q", 32 + n * bpn, n, medoid, bpn))
    Xh = np.ascontiguousarray(X, dtype=np.float16)
    for i in range(n):
        out += Xh[i].tobytes() + bytes([int(counts[i])]) + \
            np.ascontiguousarray(edges[i], np.uint32).tobytes() + \
            np.ascontiguousarray(edist[i], np.uint16).tobytes()
    flags = (1 if packed is not None else 0) | (2 if cent is not None else 0) | \
        (4 if nrm is not None else 0)
    out += struct.pack("<IIB", 0x484C5344, 1, flags)
    if packed is not None:
        ps = packed.dtype.itemsize
        out += struct.pack("<BB", k_ranks, ps)
        out += np.asarray(c, np.float32).tobytes() + np.float32(norm_denom).tobytes()
        rec = R * k_ranks * ps + 2 * R
        pad = (rec + 3) // 4 * 4 - rec
        for i in range(n):
            out += packed[i].tobytes() + mag[i].tobytes() + b"\0" * pad
    if cent is not None:
        M, K, dsub = cent.shape
        out += struct.pack("<III", M, K, dsub) + cent.astype(np.float32).tobytes()
        rec = R * M
        pad = (rec + 3) // 4 * 4 - rec
        for i in range(n):
            out += codes[i].tobytes() + b"\0" * pad
    if nrm is not None:
        out += np.asarray(nrm, np.float32).tobytes()
    with open(path, "wb") as f:
        f.write(bytes(out))


def read_directional_file(path, dim, R):
    """Reads a graph file with the full base layout (records with ids,
    deletion bitmask, next_id; graph.cuh:1653-1788) and, if present, the
    directional trailer behind it (graph.cuh:1814-1937).  Returns (rows
    [n, dim] fp16, edges [n, R] u32, bf16 edge distances [n, R] u16, counts
    [n] u8, medoid, pq) with pq = {"centroids": [M, K, dsub] f32, "codes":
    [n, R*M] u8} or None."""
    raw = open(path, "rb").read()
    _, n, medoid, bpn = struct.unpack_from("<4Q", raw, 0)
    if bpn != 2 * dim + 1 + 6 * R + 4:
        raise ValueError(f"bytes_per_node {bpn} is not the full layout for dim={dim}, R={R}")
    rec = np.frombuffer(raw, np.uint8, count=n * bpn, offset=32).reshape(n, bpn)
    rows = rec[:, :2 * dim].copy().view(np.float16)
    counts = rec[:, 2 * dim].copy()
    o = 2 * dim + 1
    edges = rec[:, o:o + 4 * R].copy().view(np.uint32)
    edist = rec[:, o + 4 * R:o + 6 * R].copy().view(np.uint16)
    off = 32 + n * bpn + (n + 7) // 8 + 8
    pq = None
    if off + 9 <= len(raw):
        magic, version, flags = struct.unpack_from("<IIB", raw, off)
        if magic == 0x484C5344:
            off += 9
            if flags & 1:
                kr, ps = struct.unpack_from("<BB", raw, off)
                off += 2 + 4 * kr + 4
                r = R * kr * ps + 2 * R
                off += n * ((r + 3) // 4 * 4)
            if flags & 2:
                M, Kc, dsub = struct.unpack_from("<III", raw, off)
                off += 12
                cent = np.frombuffer(raw, np.float32, count=M * Kc * dsub,
                                     offset=off).reshape(M, Kc, dsub).copy()
                off += 4 * M * Kc * dsub
                r = R * M
                rp = (r + 3) // 4 * 4
                codes = np.frombuffer(raw, np.uint8, count=n * rp, offset=off).reshape(n, rp)
                pq = {"centroids": cent, "codes": codes[:, :r].copy()}
    return rows, edges, edist, counts, int(medoid), pq
