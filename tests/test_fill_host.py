"""The synthetic-input generator's CPU restatement (orc_fill_normal, the
oracle's copy of v7g_fill_normal): against a float64 Box-Muller of the same
counter-based uniforms, and its distribution.  The device generator is checked
against it bit for bit in tests/test_fill_gpu.py."""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xbf58476d1ce4e5b9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94d049bb133111eb)
    return z ^ (z >> np.uint64(31))


def box_muller64(rows: int, n: int, row0: int, seed: int) -> np.ndarray:
    """float64 N(0, 1) from the generator's counter hash (SplitMix64 finaliser)."""
    with np.errstate(over="ignore"):
        key = mix64(np.array([seed], np.uint64) ^ np.uint64(0x9e3779b97f4a7c15))[0]
        r = (np.arange(rows, dtype=np.uint64) + np.uint64(row0))[:, None]
        c = np.arange(n, dtype=np.uint64)[None, :]
        h = mix64(key ^ mix64(r * np.uint64(0xd1b54a32d192ed03) + c))
    u1 = ((h >> np.uint64(40)).astype(np.float64) + 1.0) * 2.0**-24
    u2 = (h & np.uint64(0xffffff)).astype(np.float64) * 2.0**-24
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def test_fill_matches_float64_box_muller(oracle):
    for rows, n, row0, seed in ((7, 1000, 0, 0), (3, 12288, 16381, 12), (64, 96, 5, 2**63 + 5)):
        z = oracle.fill_normal(rows, n, row0, seed, 0.0, 1.0).astype(np.float64)
        ref = box_muller64(rows, n, row0, seed)
        err = np.abs(z - ref)
        assert (err <= 2e-6 * (1.0 + np.abs(ref))).all(), err.max()


def test_fill_mean_std_and_shards(oracle):
    x = oracle.fill_normal(256, 12288, 0, 13, 0.0, 2.0)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 2.0) < 0.01
    assert abs(float(((x / 2.0) ** 4).mean()) - 3.0) < 0.05  # normal kurtosis
    assert np.isfinite(x).all()
    # any row shard regenerates the same rows
    assert np.array_equal(oracle.fill_normal(10, 12288, 100, 13, 0.0, 2.0), x[100:110])
    y = oracle.fill_normal(4, 64, 0, 3, 1.0, 0.1)
    z = oracle.fill_normal(4, 64, 0, 3, 0.0, 1.0)
    assert np.array_equal(y, (np.float32(1.0) + np.float32(0.1) * z).astype(np.float32))
