"""CPU oracle for the gs2d path (TEST INFRASTRUCTURE: only tests/, smoke() and bench.py's CPU
baseline may use it; the product never does).

A numpy restatement of the toy2d reference:
  bin_gaussians   toy2d/gs2d/binning.py:35-88 (float32 rect arithmetic, stable depth argsort,
                  key tile * n + rank, ranges, bucket tables)
  forward         toy2d/csrc/rasterize.cu:106-177 (per tile, pixels vectorised, splats in list order;
                  bucket_state written per 32-splat bucket for every 256-splat round the block runs,
                  the block stopping at a round boundary once every pixel is done)
  backward        toy2d/csrc/rasterize.cu:182-258 / tests/kernel_emulator.py:92-123 (per pixel, back to
                  front, T recovered by division) - the gradient both GPU backward modes must match

Pinned against the reference itself: tests/golden/gs2d_*.npz hold outputs of the reference's own
bin_gaussians, render_reference + autograd and kernel_emulator on its test scenes and on config C1,
written by tests/golden/make_gs2d_golden.py; tests/test_gs2d_oracle.py checks this file against them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TILE = 16
BLOCK = TILE * TILE
BUCKET = 32
ALPHA_MIN = 1.0 / 255.0
ALPHA_MAX = 0.99
T_MIN = 1e-4


@dataclass
class Bins:
    H: int
    W: int
    tiles_x: int
    tiles_y: int
    rect: np.ndarray
    order: np.ndarray
    point_list: np.ndarray
    ranges: np.ndarray
    bucket_offsets: np.ndarray
    bucket_to_tile: np.ndarray
    num_buckets: int


def bin_gaussians(means, radii, depth, H: int, W: int) -> Bins:
    """binning.py:35-88. means are rounded to float32 and the rect is computed in float32 exactly
    as torch evaluates it: trunc((m - r) / 16), trunc((((m + r) + 16) - 1) / 16), clamp, to int."""
    m = np.asarray(means, dtype=np.float32).reshape(-1, 2)
    r = np.asarray(radii).astype(np.int64)
    rf = r.astype(np.float32)
    n = m.shape[0]
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = tiles_x * tiles_y
    sixteen, one = np.float32(16), np.float32(1)

    def lo(c, hi):
        v = np.trunc((m[:, c] - rf) / sixteen)
        return np.clip(v, np.float32(0), np.float32(hi)).astype(np.int64)

    def up(c, hi):
        v = np.trunc((((m[:, c] + rf) + sixteen) - one) / sixteen)
        return np.clip(v, np.float32(0), np.float32(hi)).astype(np.int64)

    xmin, ymin, xmax, ymax = lo(0, tiles_x), lo(1, tiles_y), up(0, tiles_x), up(1, tiles_y)
    valid = r > 0
    w = np.where(valid, xmax - xmin, 0)
    h = np.where(valid, ymax - ymin, 0)
    counts = np.clip(w * h, 0, None)
    empty = counts == 0
    xmax = np.where(empty, xmin, xmax)
    ymax = np.where(empty, ymin, ymax)
    rect = np.stack([xmin, ymin, xmax, ymax], axis=-1).astype(np.int32)

    d = np.asarray(depth)
    order = np.argsort(d, kind="stable").astype(np.int64)
    rank = np.empty(n, dtype=np.int64)
    rank[order] = np.arange(n)

    M = int(counts.sum())
    if M > 0:
        gid = np.repeat(np.arange(n), counts)
        first = np.cumsum(counts) - counts
        k = np.arange(M) - np.repeat(first, counts)
        wg = w[gid]
        tile = (ymin[gid] + k // wg) * tiles_x + (xmin[gid] + k % wg)
        key = tile * n + rank[gid]
        perm = np.argsort(key, kind="stable")
        point_list = gid[perm].astype(np.int32)
        per_tile = np.bincount(tile[perm], minlength=T)
    else:
        point_list = np.zeros(0, np.int32)
        per_tile = np.zeros(T, np.int64)
    start = np.cumsum(per_tile) - per_tile
    ranges = np.stack([start, start + per_tile], axis=-1).astype(np.int32)
    nb = (per_tile + BUCKET - 1) // BUCKET
    bucket_offsets = (np.cumsum(nb) - nb).astype(np.int32)
    bucket_to_tile = np.repeat(np.arange(T), nb).astype(np.int32)
    return Bins(H, W, tiles_x, tiles_y, rect, order, point_list, ranges, bucket_offsets, bucket_to_tile,
                int(nb.sum()))


@dataclass
class Forward:
    out: np.ndarray          # (3, H, W)
    final_T: np.ndarray      # (H, W)
    n_contrib: np.ndarray    # (H, W) int32
    bucket_state: np.ndarray  # (B, 256, 4) = (T, C)
    near: np.ndarray         # (H, W) bool: a decision of this pixel sat within 1e-5 (relative) of a threshold


def _tile_pixels(tile, b: Bins):
    tx, ty = tile % b.tiles_x, tile // b.tiles_x
    tid = np.arange(BLOCK)
    return tx * TILE + tid % TILE, ty * TILE + tid // TILE


def forward(means, conic, color, opacity, bg, b: Bins, dtype=np.float64) -> Forward:
    """rasterize.cu:106-177, one tile at a time, the tile's 256 pixels as one vector."""
    m = np.asarray(means, dtype).reshape(-1, 2)
    con = np.asarray(conic, dtype).reshape(-1, 3)
    col = np.asarray(color, dtype).reshape(-1, 3)
    op = np.asarray(opacity, dtype).reshape(-1)
    bgv = np.asarray(bg, dtype).reshape(3)
    H, W = b.H, b.W
    out = np.zeros((3, H, W), dtype)
    final_T = np.zeros((H, W), dtype)
    n_contrib = np.zeros((H, W), np.int32)
    near_img = np.zeros((H, W), bool)
    bstate = np.zeros((b.num_buckets, BLOCK, 4), dtype)
    amin, amax, tmin, half = dtype(ALPHA_MIN), dtype(ALPHA_MAX), dtype(T_MIN), dtype(0.5)
    one = dtype(1)
    for tile in range(b.tiles_x * b.tiles_y):
        px, py = _tile_pixels(tile, b)
        inside = (px < W) & (py < H)
        fpx, fpy = px.astype(dtype), py.astype(dtype)
        s, e = int(b.ranges[tile, 0]), int(b.ranges[tile, 1])
        todo = e - s
        bbase = int(b.bucket_offsets[tile]) if b.num_buckets else 0
        T = np.ones(BLOCK, dtype)
        C = np.zeros((BLOCK, 3), dtype)
        last = np.zeros(BLOCK, np.int32)
        done = ~inside
        near = np.zeros(BLOCK, bool)
        rounds = (todo + BLOCK - 1) // BLOCK
        for r in range(rounds):
            if done.all():
                break
            for j in range(min(BLOCK, todo - r * BLOCK)):
                idx = r * BLOCK + j
                if idx % BUCKET == 0:
                    bstate[bbase + idx // BUCKET] = np.concatenate([T[:, None], C], axis=1)
                g = int(b.point_list[s + idx])
                dx = m[g, 0] - fpx
                dy = m[g, 1] - fpy
                power = -half * (con[g, 0] * dx * dx + con[g, 2] * dy * dy) - con[g, 1] * dx * dy
                live = ~done & (power <= 0)
                with np.errstate(over="ignore"):
                    G = np.exp(np.minimum(power, 0))
                a = op[g] * G
                alpha = np.minimum(amax, a)
                near |= live & ((np.abs(a - amin) < 1e-5 * amin) | (np.abs(a - amax) < 1e-5 * amax))
                ok = live & (alpha >= amin)
                test_T = T * (one - alpha)
                near |= ok & (np.abs(test_T - tmin) < 1e-5 * tmin)
                term = ok & (test_T < tmin)
                done = done | term
                inc = ok & ~term
                w = alpha * T
                C = np.where(inc[:, None], C + col[g][None, :] * w[:, None], C)
                T = np.where(inc, test_T, T)
                last = np.where(inc, idx + 1, last)
        ys, xs = py[inside], px[inside]
        for ch in range(3):
            out[ch, ys, xs] = (C[:, ch] + T * bgv[ch])[inside]
        final_T[ys, xs] = T[inside]
        n_contrib[ys, xs] = last[inside]
        near_img[ys, xs] = near[inside]
    return Forward(out, final_T, n_contrib, bstate, near_img)


def backward(means, conic, color, opacity, bg, b: Bins, fwd: Forward, dout):
    """dL/d(means, conic, color, opacity) for upstream dout (3, H, W): rasterize.cu:182-258 per pixel."""
    dtype = np.float64
    m = np.asarray(means, dtype).reshape(-1, 2)
    con = np.asarray(conic, dtype).reshape(-1, 3)
    col = np.asarray(color, dtype).reshape(-1, 3)
    op = np.asarray(opacity, dtype).reshape(-1)
    bgv = np.asarray(bg, dtype).reshape(3)
    d = np.asarray(dout, dtype)
    H, W = b.H, b.W
    n = m.shape[0]
    dm = np.zeros((n, 2))
    dcon = np.zeros((n, 3))
    dcol = np.zeros((n, 3))
    dop = np.zeros(n)
    for tile in range(b.tiles_x * b.tiles_y):
        px, py = _tile_pixels(tile, b)
        inside = (px < W) & (py < H)
        pxc, pyc = np.minimum(px, W - 1), np.minimum(py, H - 1)
        fpx, fpy = px.astype(dtype), py.astype(dtype)
        s, e = int(b.ranges[tile, 0]), int(b.ranges[tile, 1])
        Tf = np.where(inside, fwd.final_T[pyc, pxc], 0.0)
        last = np.where(inside, fwd.n_contrib[pyc, pxc], 0)
        dp = np.where(inside[:, None], d[:, pyc, pxc].T, 0.0)
        bg_dot = dp @ bgv
        T = Tf.copy()
        acc = np.zeros((BLOCK, 3))
        la = np.zeros(BLOCK)
        lc = np.zeros((BLOCK, 3))
        for idx in range(e - s - 1, -1, -1):
            active = inside & (idx < last)
            if not active.any():
                continue
            g = int(b.point_list[s + idx])
            dx = m[g, 0] - fpx
            dy = m[g, 1] - fpy
            power = -0.5 * (con[g, 0] * dx * dx + con[g, 2] * dy * dy) - con[g, 1] * dx * dy
            G = np.exp(np.minimum(power, 0))
            a = op[g] * G
            clamped = a > ALPHA_MAX
            alpha = np.minimum(ALPHA_MAX, a)
            ok = active & (power <= 0) & (alpha >= ALPHA_MIN)
            if not ok.any():
                continue
            one_minus = 1.0 - alpha
            T = np.where(ok, T / one_minus, T)
            acc = np.where(ok[:, None], la[:, None] * lc + (1.0 - la[:, None]) * acc, acc)
            la = np.where(ok, alpha, la)
            lc = np.where(ok[:, None], col[g][None, :], lc)
            dL_dalpha = ((col[g][None, :] - acc) * dp).sum(1) * T + (-Tf / one_minus) * bg_dot
            wgt = np.where(ok, alpha * T, 0.0)
            dcol[g] += (wgt[:, None] * dp).sum(0)
            chain = ok & ~clamped
            dpow = np.where(chain, op[g] * G * dL_dalpha, 0.0)
            dop[g] += np.where(chain, G * dL_dalpha, 0.0).sum()
            dm[g, 0] += ((-con[g, 0] * dx - con[g, 1] * dy) * dpow).sum()
            dm[g, 1] += ((-con[g, 2] * dy - con[g, 1] * dx) * dpow).sum()
            dcon[g, 0] += (-0.5 * dx * dx * dpow).sum()
            dcon[g, 1] += (-dx * dy * dpow).sum()
            dcon[g, 2] += (-0.5 * dy * dy * dpow).sum()
    return dm, dcon, dcol, dop


def rel_err(a, b) -> float:
    """Norm-based relative error (toy2d/tests/scenes.py:37-39): ||a - b|| / max(||b||, 1e-30)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
