"""CPU oracle for the integer half of the 3DGS path (TEST INFRASTRUCTURE only): which tiles each Gaussian
is listed in, the 64-bit keys, their stable sort, the tile ranges and the bucket tables.

Given the per-Gaussian outputs of a preprocess (mean2d, conic, thr = ln(255 opacity), culling rectangle,
depth), it recomputes in numpy float32, operation for operation as the device does (every product and sum
rounded on its own, no fused multiply-add):
  tile test     the rectangle minimum of q = A dx^2 + 2B dx dy + C dy^2 over the tile's pixel-centre
                rectangle against 2 thr (csrc/gs3d_common.cuh, rect_min_quadratic / tile_hit)
  keys          (tile << 32) | float32 bits of the depth, generated Gaussian by Gaussian, tiles row-major
  sort          stable by key (so ties keep Gaussian order)
  ranges        per-tile [start, end) of the sorted keys; buckets = ceil(len / 32)
so the device's integer outputs must match it bit for bit. Parity of this path is UNPINNED against the
reference (Faster-GS's create_instances_cu / CUB sorts are not vendored); it restates the key layout the
benchmark spec prescribes (64-bit tile|depth keys, one radix sort).
"""
from __future__ import annotations

import numpy as np

TILE = 16
f32 = np.float32


def _quad(A, B, C, dx, dy):
    t0 = (A * dx) * dx
    t1 = ((f32(2) * B) * dx) * dy
    t2 = (C * dy) * dy
    return (t0 + t1) + t2


def tile_hits(mx, my, A, B, C, thr, tx, ty, W: int, H: int) -> np.ndarray:
    """Vectorised tile test; all float arguments float32 arrays of one shape."""
    px0 = (tx * TILE).astype(f32) + f32(0.5)
    px1 = np.minimum((tx + 1) * TILE, W).astype(f32) - f32(0.5)
    py0 = (ty * TILE).astype(f32) + f32(0.5)
    py1 = np.minimum((ty + 1) * TILE, H).astype(f32) - f32(0.5)
    x0, x1, y0, y1 = px0 - mx, px1 - mx, py0 - my, py1 - my
    in_x = (x0 <= 0) & (x1 >= 0)
    in_y = (y0 <= 0) & (y1 >= 0)
    with np.errstate(all="ignore"):
        dxe = np.where(x0 > 0, x0, x1)
        dye_ = np.minimum(np.maximum((-B * dxe) / C, y0), y1)
        q1 = np.where(in_x, f32(np.inf), _quad(A, B, C, dxe, dye_))
        dye = np.where(y0 > 0, y0, y1)
        dxe_ = np.minimum(np.maximum((-B * dye) / A, x0), x1)
        q2 = np.where(in_y, f32(np.inf), _quad(A, B, C, dxe_, dye))
    q = np.where(in_x & in_y, f32(0), np.minimum(q1, q2))
    return q <= f32(2) * thr


def bin_instances(mean2d, conic_o, thr, rect, depth, visible, W: int, H: int):
    """(n_touched [N], keys [M] uint64 in generation order, ids [M], keys_sorted, point_list, ranges [T,2],
    bucket counts [T]) for the visible Gaussians."""
    mean2d = np.asarray(mean2d, f32)
    conic_o = np.asarray(conic_o, f32)
    thr = np.asarray(thr, f32)
    rect = np.asarray(rect).astype(np.int64)
    depth = np.asarray(depth, f32)
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = tiles_x * tiles_y
    n = mean2d.shape[0]
    ids_all, tx_all, ty_all = [], [], []
    vis = np.nonzero(np.asarray(visible))[0]
    for i in vis:  # Gaussian order, tiles row-major: the device's generation order
        x0, y0, x1, y1 = rect[i]
        tys, txs = np.meshgrid(np.arange(y0 // TILE, y1 // TILE + 1), np.arange(x0 // TILE, x1 // TILE + 1),
                               indexing="ij")
        tx_all.append(txs.ravel())
        ty_all.append(tys.ravel())
        ids_all.append(np.full(txs.size, i))
    n_touched = np.zeros(n, np.int64)
    if not ids_all:
        return (n_touched, np.zeros(0, np.uint64), np.zeros(0, np.int64), np.zeros(0, np.uint64),
                np.zeros(0, np.int64), np.zeros((T, 2), np.int64), np.zeros(T, np.int64))
    ids = np.concatenate(ids_all)
    tx = np.concatenate(tx_all)
    ty = np.concatenate(ty_all)
    hit = tile_hits(mean2d[ids, 0], mean2d[ids, 1], conic_o[ids, 0], conic_o[ids, 1], conic_o[ids, 2], thr[ids], tx,
                    ty, W, H)
    ids, tx, ty = ids[hit], tx[hit], ty[hit]
    np.add.at(n_touched, ids, 1)
    tile = (ty * tiles_x + tx).astype(np.uint64)
    keys = (tile << np.uint64(32)) | depth[ids].view(np.uint32).astype(np.uint64)
    perm = np.argsort(keys, kind="stable")
    keys_sorted = keys[perm]
    point_list = ids[perm]
    t_sorted = (keys_sorted >> np.uint64(32)).astype(np.int64)
    counts = np.bincount(t_sorted, minlength=T)
    ranges = np.zeros((T, 2), np.int64)
    first = np.searchsorted(t_sorted, np.arange(T), side="left")
    last = np.searchsorted(t_sorted, np.arange(T), side="right")
    nonempty = counts > 0
    ranges[nonempty, 0] = first[nonempty]
    ranges[nonempty, 1] = last[nonempty]
    buckets = (counts + 31) // 32
    return n_touched, keys, ids, keys_sorted, point_list, ranges, buckets
