"""The int8 quantizer's division-free rounding, emulated in float32 on the CPU.

The device quantizer (kv_cache_bench_b200/csrc/kvb_pages.cu: quantize4_fast / quantize4_exact)
computes t = x * fl(1 / scale), rounds t with the 1.5 * 2^23 bias, and falls back to the IEEE division
of the reference (src/reference.cpp:32-51: nearbyint(x / scale)) only when t lies within 2^-14 of a
half-integer. These tests restate that rule step by step in numpy float32 and check it against the
division on random pages of many magnitudes and on planted exact ties (x = (k + 1/2) * scale), where
a wrong rule would show first. The GPU tests check the kernel itself bit for bit against the oracle.
"""
import numpy as np

MAGIC = np.float32(12582912.0)  # 1.5 * 2^23
NEAR = np.float32(0.5) - np.float32(2.0 ** -14)


def fast_rule(x, scale):
    rcp = np.float32(1.0) / scale
    t = (x * rcp).astype(np.float32)
    y = (t + MAGIC).astype(np.float32)
    q = y.view(np.int32) - 0x4B400000
    near = np.abs((t - (y - MAGIC).astype(np.float32)).astype(np.float32)) >= NEAR
    exact = np.rint((x / scale).astype(np.float32)).astype(np.int32)
    return np.clip(np.where(near, exact, q), -127, 127), near


def reference_rule(x, scale):
    return np.clip(np.rint((x / scale).astype(np.float32)), -127, 127).astype(np.int32)


def test_fast_rounding_equals_the_division():
    rng = np.random.default_rng(7)
    total = near_total = 0
    for _ in range(60):
        amax = np.float32(10.0 ** rng.uniform(-30, 30))
        scale = np.float32(amax / np.float32(127))
        x = (rng.uniform(-1, 1, 50_000).astype(np.float32) * amax).astype(np.float32)
        k = rng.integers(-127, 127, 500)
        ties = ((k + 0.5) * np.float64(scale)).astype(np.float32)
        x = np.concatenate([x, ties[np.abs(ties) <= amax], np.array([amax, -amax, 0.0], np.float32)])
        got, near = fast_rule(x, scale)
        assert np.array_equal(got, reference_rule(x, scale))
        total += x.size
        near_total += int(near.sum())
    # the fallback stays rare: mostly the planted ties
    assert near_total < 0.05 * total
