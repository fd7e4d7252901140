"""CPU restatement of the reference's lean Adam (TEST INFRASTRUCTURE only; never called by the product path).

Follows `adam_step_sparse_cu<LOWP>` of cluster/patches/fastergs_lean_adam.patch:72-130:
  hash_u32 (:72-75)      the lowbias32 integer hash (C. Wellons), two multiply-xorshift rounds
  bf16 read (:77-79)     bits << 16
  SR write (:83-86)      (bits(f) + (rnd & 0xFFFF)) >> 16, rnd = hash((uint32) i ^ seed) for exp_avg and
                         hash of that for exp_avg_sq (:122-123), seed = 0x9E3779B9 * step + 0x85EBCA6B (:165)
  update (:116-120)      m = fma(b1, m - g, g); v = fma(b2, v - g^2, g^2); p -= step_size * m / fma(sqrt(v), bc2, eps)
  mask (:106)            element i is skipped when visibility[i // features] == 0
numpy uint32 arithmetic wraps like the device's. The update below uses float64 for the fused multiply-adds, which
is exact for the products and can differ from a float32 fma in the last bit of the sum, so parity tests compare the
update with a tolerance and the rounding (the integer part) bit for bit.
"""
from __future__ import annotations

import numpy as np

U32 = np.uint32


def lowbias32(x) -> np.ndarray:
    x = np.asarray(x, dtype=U32).copy()
    x ^= x >> U32(16)
    x *= U32(0x7FEB352D)
    x ^= x >> U32(15)
    x *= U32(0x846CA68B)
    x ^= x >> U32(16)
    return x


def seed_for_step(step: int) -> np.uint32:
    return U32((0x9E3779B9 * step + 0x85EBCA6B) & 0xFFFFFFFF)


def bf16_bits_to_float(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(U32) << U32(16)).view(np.float32)


def float_to_bf16_bits_sr(f, rnd) -> np.ndarray:
    u = np.asarray(f, dtype=np.float32).view(U32)
    return ((u + (np.asarray(rnd, dtype=U32) & U32(0xFFFF))) >> U32(16)).astype(np.uint16)


def sr_randoms(n: int, step: int) -> tuple[np.ndarray, np.ndarray]:
    """(r1, r2) for elements 0..n-1 of a group at this step."""
    r1 = lowbias32(np.arange(n, dtype=np.uint64).astype(U32) ^ seed_for_step(step))
    return r1, lowbias32(r1)


def adam_lean(param, grad, m, v, step: int, lr: float, beta1=0.9, beta2=0.999, eps=1e-15, visibility=None,
              features: int = 1, lowp: bool = False):
    """One lean step on flat float32 arrays (m, v float32, or uint16 bf16 bits when lowp). Returns new copies."""
    p = np.asarray(param, np.float32).copy()
    g = np.asarray(grad, np.float32)
    mf = bf16_bits_to_float(m) if lowp else np.asarray(m, np.float32)
    vf = bf16_bits_to_float(v) if lowp else np.asarray(v, np.float32)
    # host arithmetic of the wrapper (:162-164): double precision, rounded once
    step_size = np.float32(lr * (1.0 / (1.0 - beta1 ** step)))
    bc2_sqrt_rcp = np.float32(1.0 / np.sqrt(1.0 - beta2 ** step))
    g2 = (g * g).astype(np.float32)
    m1 = (np.float64(np.float32(beta1)) * (mf - g).astype(np.float64) + g).astype(np.float32)
    m2 = (np.float64(np.float32(beta2)) * (vf - g2).astype(np.float64) + g2).astype(np.float32)
    denom = (np.sqrt(m2).astype(np.float64) * np.float64(bc2_sqrt_rcp) + np.float64(np.float32(eps))).astype(np.float32)
    upd = (p - step_size * m1 / denom).astype(np.float32)
    on = np.ones(p.shape, bool) if visibility is None else (np.asarray(visibility)[np.arange(p.size) // features] != 0)
    p = np.where(on, upd, p)
    if lowp:
        r1, r2 = sr_randoms(p.size, step)
        m_out = np.where(on, float_to_bf16_bits_sr(m1, r1), np.asarray(m, np.uint16))
        v_out = np.where(on, float_to_bf16_bits_sr(m2, r2), np.asarray(v, np.uint16))
    else:
        m_out = np.where(on, m1, mf)
        v_out = np.where(on, m2, vf)
    return p, m_out, v_out
