"""CPU oracle for the splat2d path (TEST INFRASTRUCTURE: only tests/, smoke() and bench.py's CPU
baseline may use it; the product never does).

A numpy restatement of phase0's splat2d:
  bin_tiles   phase0/splat2d/ops.py:206-255 (float64 alpha >= 1/255 ellipse bbox, +-1 px, CSR lists)
  forward     phase0/csrc/macrotile/splat2d_cpu.cpp:317-358 (T checked before each splat; checkpoint
              (C, T) at every bucket start; n_contrib = count, last_contrib = position + 1)
  backward    splat2d_cpu.cpp:360-390 (per pixel, back to front from last_contrib, T by division),
              chain rule splat2d_common.h:227-246 - the gradient both GPU backward modes must match

Pinned against the reference itself: tests/golden/splat2d_*.npz hold the reference's bin_tiles,
ref_render + autograd and its compiled CPU extension (oracle/_ref) outputs for the reference's own
gradcheck scenes (phase0/tests/gradcheck/conftest.py), written by tests/golden/make_splat2d_golden.py;
tests/test_splat2d_oracle.py checks this file against them and against oracle/_ref when it is built.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TILE = 16
BLOCK = TILE * TILE
BUCKET = 32
ALPHA_MIN = 1.0 / 255.0
ALPHA_MAX = 0.99
T_STOP = 1e-4


@dataclass
class TileBins:
    tile_offsets: np.ndarray
    tile_ids: np.ndarray
    bucket_offsets: np.ndarray
    bucket_tile: np.ndarray
    tiles_x: int
    tiles_y: int

    @property
    def num_buckets(self) -> int:
        return int(self.bucket_tile.size)


def bin_tiles(means, chol, opacity_logit, H: int, W: int) -> TileBins:
    m = np.asarray(means, np.float64).reshape(-1, 2)
    lc = np.asarray(chol, np.float64).reshape(-1, 3)
    o = 1.0 / (1.0 + np.exp(-np.asarray(opacity_logit, np.float64).reshape(-1)))
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    with np.errstate(divide="ignore", invalid="ignore"):
        r2 = 2.0 * np.log(255.0 * o)
        r = np.sqrt(np.clip(r2, 0.0, None))
        l0, l1, l2 = lc[:, 0], lc[:, 1], lc[:, 2]
        ex = r * np.sqrt(1.0 / l0**2 + (l1 / (l0 * l2)) ** 2)
        ey = r / np.abs(l2)
    x0 = np.floor(m[:, 0] - ex - 0.5) - 1
    x1 = np.ceil(m[:, 0] + ex - 0.5) + 1
    y0 = np.floor(m[:, 1] - ey - 0.5) - 1
    y1 = np.ceil(m[:, 1] + ey - 0.5) + 1
    valid = (r2 > 0) & (x1 >= 0) & (x0 <= W - 1) & (y1 >= 0) & (y0 <= H - 1)
    tx0 = np.floor(np.clip(x0, 0, W - 1) / TILE)
    tx1 = np.floor(np.clip(x1, 0, W - 1) / TILE)
    ty0 = np.floor(np.clip(y0, 0, H - 1) / TILE)
    ty1 = np.floor(np.clip(y1, 0, H - 1) / TILE)
    lists = []
    for ty in range(tiles_y):
        for tx in range(tiles_x):
            hit = valid & (tx0 <= tx) & (tx1 >= tx) & (ty0 <= ty) & (ty1 >= ty)
            lists.append(np.nonzero(hit)[0])
    counts = np.array([len(x) for x in lists], np.int64)
    tile_offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    tile_ids = (np.concatenate(lists) if lists else np.zeros(0)).astype(np.int32)
    nb = (counts + BUCKET - 1) // BUCKET
    bucket_offsets = np.concatenate([[0], np.cumsum(nb)]).astype(np.int32)
    bucket_tile = np.repeat(np.arange(len(lists)), nb).astype(np.int32)
    return TileBins(tile_offsets, tile_ids, bucket_offsets, bucket_tile, tiles_x, tiles_y)


@dataclass
class Forward:
    image: np.ndarray        # (H, W, 3)
    t_final: np.ndarray      # (H, W)
    n_contrib: np.ndarray    # (H, W) int32
    last_contrib: np.ndarray  # (H, W) int32
    ckpt: np.ndarray         # (B, 256, 4) = (C, T)


def _pixels(tile, tiles_x):
    lane = np.arange(BLOCK)
    return (tile % tiles_x) * TILE + lane % TILE, (tile // tiles_x) * TILE + lane // TILE


def _eval(m, l, o, px, py):
    dx = px - m[0]
    dy = py - m[1]
    a = l[0] * dx + l[1] * dy
    b = l[2] * dy
    g = np.exp(-0.5 * (a * a + b * b))
    raw = o * g
    clamped = raw > ALPHA_MAX
    return dx, dy, a, b, g, np.where(clamped, ALPHA_MAX, raw), clamped


def forward(means, chol, opacity_logit, colors, bins: TileBins, H: int, W: int) -> Forward:
    m = np.asarray(means, np.float64).reshape(-1, 2)
    lc = np.asarray(chol, np.float64).reshape(-1, 3)
    o = 1.0 / (1.0 + np.exp(-np.asarray(opacity_logit, np.float64).reshape(-1)))
    col = np.asarray(colors, np.float64).reshape(-1, 3)
    image = np.zeros((H, W, 3))
    t_final = np.ones((H, W))
    n_contrib = np.zeros((H, W), np.int32)
    last_contrib = np.zeros((H, W), np.int32)
    ckpt = np.zeros((bins.num_buckets, BLOCK, 4))
    for tile in range(bins.tiles_x * bins.tiles_y):
        x, y = _pixels(tile, bins.tiles_x)
        inside = (x < W) & (y < H)
        px, py = x + 0.5, y + 0.5
        C = np.zeros((BLOCK, 3))
        T = np.ones(BLOCK)
        cnt = np.zeros(BLOCK, np.int32)
        last = np.zeros(BLOCK, np.int32)
        s, e = int(bins.tile_offsets[tile]), int(bins.tile_offsets[tile + 1])
        b0 = int(bins.bucket_offsets[tile])
        for local in range(e - s):
            if local % BUCKET == 0:
                ckpt[b0 + local // BUCKET] = np.concatenate([C, T[:, None]], axis=1)
            g = int(bins.tile_ids[s + local])
            live = inside & ~(T < T_STOP)
            _, _, _, _, _, alpha, _ = _eval(m[g], lc[g], o[g], px, py)
            ok = live & (alpha >= ALPHA_MIN)
            C = np.where(ok[:, None], C + col[g][None, :] * (alpha * T)[:, None], C)
            T = np.where(ok, T * (1.0 - alpha), T)
            cnt += ok
            last = np.where(ok, local + 1, last)
        ys, xs = y[inside], x[inside]
        image[ys, xs] = C[inside]
        t_final[ys, xs] = T[inside]
        n_contrib[ys, xs] = cnt[inside]
        last_contrib[ys, xs] = last[inside]
    return Forward(image, t_final, n_contrib, last_contrib, ckpt)


def backward(grad_image, means, chol, opacity_logit, colors, bins: TileBins, H: int, W: int, fwd: Forward):
    """Gradients (means, chol, opacity_logit, colors) for grad_image [H, W, 3]."""
    m = np.asarray(means, np.float64).reshape(-1, 2)
    lc = np.asarray(chol, np.float64).reshape(-1, 3)
    o = 1.0 / (1.0 + np.exp(-np.asarray(opacity_logit, np.float64).reshape(-1)))
    col = np.asarray(colors, np.float64).reshape(-1, 3)
    G_img = np.asarray(grad_image, np.float64)
    n = m.shape[0]
    gm, gc, gz, gcol = np.zeros((n, 2)), np.zeros((n, 3)), np.zeros(n), np.zeros((n, 3))
    for tile in range(bins.tiles_x * bins.tiles_y):
        x, y = _pixels(tile, bins.tiles_x)
        inside = (x < W) & (y < H)
        xc, yc = np.minimum(x, W - 1), np.minimum(y, H - 1)
        px, py = x + 0.5, y + 0.5
        G = np.where(inside[:, None], G_img[yc, xc], 0.0)
        T_after = np.where(inside, fwd.t_final[yc, xc], 1.0)
        last = np.where(inside, fwd.last_contrib[yc, xc], 0)
        S_acc = np.zeros((BLOCK, 3))
        s, e = int(bins.tile_offsets[tile]), int(bins.tile_offsets[tile + 1])
        for local in range(e - s - 1, -1, -1):
            active = local < last
            if not active.any():
                continue
            g = int(bins.tile_ids[s + local])
            dx, dy, a, b, gauss, alpha, clamped = _eval(m[g], lc[g], o[g], px, py)
            ok = active & (alpha >= ALPHA_MIN)
            if not ok.any():
                continue
            one_minus = 1.0 - alpha
            T = T_after / one_minus
            dL_dc = G * (alpha * T)[:, None]
            dot = (G * (col[g][None, :] - S_acc)).sum(1)
            S_acc = np.where(ok[:, None], alpha[:, None] * col[g][None, :] + one_minus[:, None] * S_acc, S_acc)
            T_after = np.where(ok, T, T_after)
            d_alpha = np.where(ok & ~clamped, T * dot, 0.0)
            d_z = d_alpha * gauss * o[g] * (1.0 - o[g])
            d_q = -0.5 * gauss * o[g] * d_alpha
            gm[g, 0] += (-d_q * 2 * a * lc[g, 0]).sum()
            gm[g, 1] += (-d_q * (2 * a * lc[g, 1] + 2 * b * lc[g, 2])).sum()
            gc[g, 0] += (d_q * 2 * a * dx).sum()
            gc[g, 1] += (d_q * 2 * a * dy).sum()
            gc[g, 2] += (d_q * 2 * b * dy).sum()
            gz[g] += d_z.sum()
            gcol[g] += np.where(ok[:, None], dL_dc, 0.0).sum(0)
    return gm, gc, gz, gcol


def rel_err(a, b) -> float:
    """Norm-based relative error (phase0/tests/gradcheck/test_gradcheck.py:24-28)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))
