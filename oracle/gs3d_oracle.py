"""CPU oracle for the integer half of the 3DGS path (TEST INFRASTRUCTURE only): which tiles each Gaussian
is listed in, the 64-bit keys, their stable sort, the tile ranges and the bucket tables.

Given the per-Gaussian outputs of a preprocess (mean2d, conic, thr = ln(255 opacity), depth), it recomputes in
numpy float32, operation for operation as the device does (every product and sum rounded on its own, no fused
multiply-add):
  listing   per tile row, the x-extent of the ellipse q = A dx^2 + 2B dx dy + C dy^2 <= 2 thr over the row's
            band of pixel centres, in closed form (csrc/gs3d_common.cuh: make_ellipse, ellipse_rows,
            ellipse_row_tiles); the tiles whose pixel-centre range meets it are listed
  keys      (tile << 32) | order-preserving bits of the depth, generated Gaussian by Gaussian (id order),
            tiles row-major
  sort      stable by key (ties keep Gaussian order)
  ranges    per-tile [start, end) of the sorted keys; buckets = ceil(len / 32)
so the device's integer outputs must match it bit for bit. Parity of this path is UNPINNED against the
reference (Faster-GS's create_instances_cu / CUB sorts are not vendored); it restates the key layout the
benchmark spec prescribes (64-bit tile|depth keys, one stable radix sort).
"""
from __future__ import annotations

import numpy as np

TILE = 16
f32 = np.float32


def depth_order_key(z) -> np.ndarray:
    """uint32 keys whose unsigned order is the float order of z."""
    b = np.asarray(z, f32).view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def _x_extent(A, B, R, D, inv_a, dy, sign):
    disc = np.maximum((A * R) - ((D * dy) * dy), f32(0))
    return ((-B) * dy + f32(sign) * np.sqrt(disc)) * inv_a


def listed_tiles(mx, my, A, B, C, thr, W: int, H: int):
    """(gaussian index, tile x, tile y) of every listing, in device generation order (Gaussian order,
    rows top to bottom, tiles left to right)."""
    mx, my, A, B, C, thr = (np.asarray(v, f32) for v in (mx, my, A, B, C, thr))
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    R = f32(2) * thr
    D = (A * C) - (B * B)
    sixteenth = f32(0.0625)
    with np.errstate(all="ignore"):
        inv_d, inv_c, inv_a = f32(1) / D, f32(1) / C, f32(1) / A  # correctly rounded reciprocals
        ey = np.sqrt((A * R) * inv_d)
        s = np.sqrt((R * inv_d) * inv_c)
        top, bot = my - ey, my + ey
        ok = (bot >= f32(0.5)) & (top <= f32(H) - f32(0.5))
        rlo = np.maximum(np.ceil((top - f32(15.5)) * sixteenth), -1).astype(np.int64)
        rhi = np.minimum(np.floor((bot - f32(0.5)) * sixteenth), tiles_y).astype(np.int64)
    rlo = np.maximum(rlo, 0)
    rhi = np.minimum(rhi, tiles_y - 1)
    nrows = np.where(ok, np.maximum(rhi - rlo + 1, 0), 0)
    g = np.repeat(np.arange(mx.size), nrows)
    ty = rlo[g] + (np.arange(g.size) - np.repeat(np.cumsum(nrows) - nrows, nrows))
    y0 = (ty * TILE).astype(f32) + f32(0.5)
    y1 = np.minimum(ty * TILE + TILE, H).astype(f32) - f32(0.5)
    with np.errstate(all="ignore"):
        lo = np.maximum(y0 - my[g], -ey[g])
        hi = np.minimum(y1 - my[g], ey[g])
        dyr = np.minimum(np.maximum((-B[g]) * s[g], lo), hi)
        dyl = np.minimum(np.maximum(B[g] * s[g], lo), hi)
        xr = mx[g] + _x_extent(A[g], B[g], R[g], D[g], inv_a[g], dyr, 1.0)
        xl = mx[g] + _x_extent(A[g], B[g], R[g], D[g], inv_a[g], dyl, -1.0)
        row_ok = (lo <= hi) & (xr >= f32(0.5)) & (xl <= f32(W) - f32(0.5))
        tlo = np.maximum(np.ceil((xl - f32(15.5)) * sixteenth), -1).astype(np.int64)
        thi = np.minimum(np.floor((xr - f32(0.5)) * sixteenth), tiles_x).astype(np.int64)
    tlo = np.maximum(tlo, 0)
    thi = np.minimum(thi, tiles_x - 1)
    ncols = np.where(row_ok, np.maximum(thi - tlo + 1, 0), 0)
    gi = np.repeat(g, ncols)
    tyi = np.repeat(ty, ncols)
    txi = np.repeat(tlo, ncols) + (np.arange(gi.size) - np.repeat(np.cumsum(ncols) - ncols, ncols))
    return gi, txi, tyi


def bin_instances(mean2d, conic_o, thr, depth, visible, W: int, H: int):
    """(n_touched [N], keys [M] uint64 in generation order, ids [M], keys_sorted, point_list, ranges [T,2],
    bucket counts [T]) for the visible Gaussians."""
    mean2d = np.asarray(mean2d, f32)
    conic_o = np.asarray(conic_o, f32)
    thr = np.asarray(thr, f32)
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = tiles_x * tiles_y
    n = mean2d.shape[0]
    vis = np.nonzero(np.asarray(visible))[0]
    gl, tx, ty = listed_tiles(mean2d[vis, 0], mean2d[vis, 1], conic_o[vis, 0], conic_o[vis, 1], conic_o[vis, 2],
                              thr[vis], W, H)
    ids = vis[gl]
    n_touched = np.bincount(ids, minlength=n).astype(np.int64)
    tile = (ty * tiles_x + tx).astype(np.uint64)
    keys = (tile << np.uint64(32)) | depth_order_key(np.asarray(depth, f32)[ids]).astype(np.uint64)
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
