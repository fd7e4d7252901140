"""The CPU restatement of the lean Adam (oracle/adam_oracle.py): hash and stochastic rounding properties."""
from __future__ import annotations

import numpy as np

from oracle import adam_oracle as O


def test_lowbias32_wraps_and_mixes():
    x = np.arange(1 << 16, dtype=np.uint32)
    h = O.lowbias32(x)
    assert h.dtype == np.uint32
    assert np.unique(h).size == x.size  # a bijection on 32-bit words
    assert O.lowbias32(np.uint32(0)) == 0  # zero is its fixed point
    bits = np.unpackbits(h.view(np.uint8)).reshape(-1, 32).mean(0)
    assert np.all(np.abs(bits - 0.5) < 0.01)


def test_sr_is_unbiased_and_brackets():
    rng = np.random.default_rng(0)
    f = rng.standard_normal(200_000).astype(np.float32)
    r1, _ = O.sr_randoms(f.size, 3)
    b = O.float_to_bf16_bits_sr(f, r1)
    down = (f.view(np.uint32) >> np.uint32(16)).astype(np.uint16)
    assert np.all((b == down) | (b == down + 1))  # rounds to one of the two neighbours
    back = O.bf16_bits_to_float(b).astype(np.float64)
    rel = (back - f) / np.abs(f)
    assert abs(rel.mean()) < 2e-4  # unbiased (truncation alone is biased by half an ulp, ~2e-3)


def test_sparse_oracle_leaves_masked_rows():
    rng = np.random.default_rng(1)
    p = rng.standard_normal(30).astype(np.float32)
    g = rng.standard_normal(30).astype(np.float32)
    vis = np.array([1, 0] * 5, np.int32)
    out = O.adam_lean(p, g, np.zeros(30, np.float32), np.zeros(30, np.float32), 1, 1e-2, visibility=vis, features=3)
    masked = np.repeat(vis == 0, 3)
    assert np.array_equal(out[0][masked], p[masked]) and np.all(out[0][~masked] != p[~masked])
