"""Shared test helpers: seeded pools, tolerances, oracle calls."""
from __future__ import annotations

import numpy as np

# Tolerances (north_star): bf16 KV max-abs 2e-2 and mean-rel 1e-3 against the
# f32 oracle on the same bf16-rounded inputs, with the oracle output rounded to
# the query dtype (ReferenceBackend returns the query's dtype). mean-rel is
# sum|a-b| / sum|b|. FP8 KV is compared with the oracle run on the
# bit-identical dequantised pages at the same bounds, and with the bf16-KV
# oracle at 1.25x the error of the oracle's own FP8 path on the same inputs
# (that own error must itself stay under the FP8_*_CAP sanity caps).
MAX_ABS = 2e-2
MEAN_REL = 1e-3
F32_MAX_ABS = 1e-4
F32_MEAN_REL = 1e-5
# Sanity caps on the oracle's own FP8 error (x50 outliers in K and V make
# per-head E4M3 / MXFP8 coarse; these only catch a broken codec).
FP8_MAX_ABS_CAP = 20.0
FP8_MEAN_REL_CAP = 0.15


def bf16_bits(x: np.ndarray) -> np.ndarray:
    from oracle import f32_to_bf16_bits

    return f32_to_bf16_bits(x)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def errors(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(got - ref)
    denom = np.abs(ref).sum()
    return float(diff.max(initial=0.0)), float(diff.sum() / denom) if denom > 0 else float(diff.sum())


def assert_close(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL, what=""):
    ma, mr = errors(got, ref)
    assert ma <= max_abs and mr <= mean_rel, f"{what}: max_abs={ma:.3e} mean_rel={mr:.3e}"
    return ma, mr


def random_pool(rng: np.random.Generator, P: int, Hkv: int, D: int, outliers: float = 0.0):
    x = rng.standard_normal((P, 2, Hkv, 16, D)).astype(np.float32)
    if outliers:
        m = rng.random(x.shape) < outliers
        x[m] *= 50.0
    return x
