"""Generates the golden fixtures in this directory (run from the repo root:
``python tests/golden/make_golden.py``).

The reference ships no known-answer vectors for this path (its attention and
quantization tests check shapes only: crates/dendrite-core/src/attention/backend.rs:376-497,
crates/dendrite-core/src/quantization/fp8.rs:183-231) and cannot be built
here, so the fixtures are computed with independent implementations of the
same definitions:

* ``fp8_codec.npz`` — FP8 E4M3 encode/decode and E8M0 decode from
  ``ml_dtypes`` (float8_e4m3fn / float8_e8m0fnu), cross-checked against
  ``torch.float8_e4m3fn``. Saturation (the reference's clamp to +-448,
  fp8.rs:130) is applied before the cast, since both libraries map
  overflow to NaN.
* ``quant_kv.npz`` — a small seeded KV pool with outliers, its per-head E4M3
  quantisation (scale = amax * f32(1/448), fp8.rs:125 via candle's affine
  divide-by-scalar; code = E4M3(clamp(x / scale))) and its MXFP8 quantisation
  (OCP MX v1.0: e = floor(log2 amax) - 8 per 32 elements), all in numpy +
  ml_dtypes.
* ``attention_small.npz`` — a seeded paged decode batch (GQA 8/2, D=64,
  non-contiguous pages, partial last pages, one empty table) and its output
  computed in float64 with torch from the definition of
  ReferenceBackend::decode (backend.rs:206-265: gather, concat, tile GQA
  h % Hkv, softmax(q k^T * scale) v).
"""
from __future__ import annotations

from pathlib import Path

import ml_dtypes
import numpy as np
import torch

HERE = Path(__file__).resolve().parent
E4M3_MAX = 448.0


def e4m3_ref(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    c = np.clip(x, -E4M3_MAX, E4M3_MAX).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
    t = torch.from_numpy(np.clip(x, -E4M3_MAX, E4M3_MAX)).to(torch.float8_e4m3fn).view(torch.uint8)
    fin = np.isfinite(x)
    assert np.array_equal(c[fin], t.numpy()[fin]), "ml_dtypes and torch disagree"
    return c


def fp8_codec(rng: np.random.Generator) -> dict:
    codes = np.arange(256, dtype=np.uint8)
    dec = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    vals = dec[np.isfinite(dec)]
    pos = np.unique(np.abs(vals))
    mids = (pos[:-1] + pos[1:]) / 2  # exact RNE ties
    near = np.concatenate([np.nextafter(mids, np.inf, dtype=np.float32),
                           np.nextafter(mids, -np.inf, dtype=np.float32)])
    edge = np.array([0.0, -0.0, 448.0, 449.0, 463.99, 464.0, 464.01, 480.0, 1e6, 3e38,
                     2.0 ** -9, 2.0 ** -10, 2.0 ** -10 * 3, 2.0 ** -11, 2.0 ** -6, 2.0 ** -7,
                     1e-30, 1e-45], dtype=np.float32)
    rnd = np.concatenate([rng.standard_normal(4000) * s for s in (1e-3, 0.05, 1.0, 30.0, 300.0)])
    x = np.concatenate([vals, mids, near, edge, rnd]).astype(np.float32)
    x = np.concatenate([x, -x]).astype(np.float32)
    e8 = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e8m0fnu).astype(np.float32)
    return {"e4m3_decode": dec, "enc_x": x, "enc_code": e4m3_ref(x), "e8m0_decode": e8}


def pool_with_outliers(rng, P, Hkv, D, frac=0.001, mult=50.0) -> np.ndarray:
    x = rng.standard_normal((P, 2, Hkv, 16, D)).astype(np.float32)
    mask = rng.random(x.shape) < frac
    x[mask] *= mult
    return x


def bf16_round(x: np.ndarray) -> np.ndarray:
    return x.astype(ml_dtypes.bfloat16)


def quant_fixture(rng) -> dict:
    P, Hkv, D = 10, 2, 64
    pool = bf16_round(pool_with_outliers(rng, P, Hkv, D, frac=0.01))
    pool_bits = pool.view(np.uint16)
    xf = pool.astype(np.float32)
    # per-head E4M3, scale = amax * f32(1/448)
    amax = np.abs(xf).max(axis=(0, 3, 4))                    # [2, Hkv]
    scale = (amax * np.float32(1.0 / 448.0)).astype(np.float32)
    scale[amax == 0] = 1.0
    q = (xf / scale[None, :, :, None, None]).astype(np.float32)
    codes_h = e4m3_ref(q)
    deq_h = (codes_h.view(ml_dtypes.float8_e4m3fn).astype(np.float32) * scale[None, :, :, None, None])
    # MXFP8 along D in blocks of 32
    blk = xf.reshape(-1, 32)
    bmax = np.abs(blk).max(axis=1)
    with np.errstate(divide="ignore"):
        e = np.where(bmax > 0, np.floor(np.log2(bmax.astype(np.float64))) - 8, -127)
    e = np.maximum(e, -127).astype(np.int32)
    codes_mx = e4m3_ref((blk * np.ldexp(np.float32(1), -e)[:, None]).astype(np.float32))
    deq_mx = codes_mx.view(ml_dtypes.float8_e4m3fn).astype(np.float32) * np.ldexp(np.float32(1), e)[:, None]
    return {
        "pool_bf16_bits": pool_bits,
        "head_scales": scale,
        "head_codes": codes_h,
        "head_deq_bf16_bits": bf16_round(deq_h.astype(np.float32)).view(np.uint16),
        "mx_codes": codes_mx.reshape(pool.shape),
        "mx_scales": (e + 127).astype(np.uint8).reshape(pool.shape[:-1] + (D // 32,)),
        "mx_deq_bf16_bits": bf16_round(deq_mx.astype(np.float32)).reshape(pool.shape).view(np.uint16),
    }


def attention_fixture(rng) -> dict:
    Hq, Hkv, D, P = 8, 2, 64, 14
    pool = rng.standard_normal((P, 2, Hkv, 16, D)).astype(np.float32)
    perm = rng.permutation(P).astype(np.uint32)
    ntok = np.array([37, 16, 1, 0, 64, 23], dtype=np.int32)
    tables, k = [], 0
    for n in ntok:
        nb = -(-int(n) // 16)
        tables.append(perm[k:k + nb])
        k += nb
    tables[1] = tables[0][:1]  # a shared first block
    indptr = np.zeros(len(ntok) + 1, dtype=np.int32)
    for i, t in enumerate(tables):
        indptr[i + 1] = indptr[i] + len(t)
    ids = np.concatenate(tables).astype(np.uint32)
    q = rng.standard_normal((len(ntok), Hq, D)).astype(np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(D))
    out = np.zeros((len(ntok), Hq, D), dtype=np.float64)
    lse = np.full((len(ntok), Hq), -np.inf)
    pt = torch.from_numpy(pool).double()
    for b, n in enumerate(ntok):
        if n == 0:
            continue
        blocks = ids[indptr[b]:indptr[b + 1]]
        K = torch.cat([pt[int(i), 0] for i in blocks], dim=1)[:, :n]  # [Hkv, T, D]
        V = torch.cat([pt[int(i), 1] for i in blocks], dim=1)[:, :n]
        K, V = K.repeat(Hq // Hkv, 1, 1), V.repeat(Hq // Hkv, 1, 1)  # tile: head h -> h % Hkv
        s = torch.einsum("hd,htd->ht", torch.from_numpy(q[b]).double(), K) * float(scale)
        lse[b] = torch.logsumexp(s, dim=-1).numpy()
        out[b] = torch.einsum("ht,htd->hd", torch.softmax(s, dim=-1), V).numpy()
    return {"pool": pool, "indptr": indptr, "block_ids": ids, "num_tokens": ntok, "q": q,
            "num_kv_heads": np.int32(Hkv), "out": out, "lse": lse}


def main() -> None:
    rng = np.random.default_rng(0xD3D1)
    np.savez_compressed(HERE / "fp8_codec.npz", **fp8_codec(rng))
    np.savez_compressed(HERE / "quant_kv.npz", **quant_fixture(rng))
    np.savez_compressed(HERE / "attention_small.npz", **attention_fixture(rng))
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
