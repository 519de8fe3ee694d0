"""CPU oracle for the cascade decode-attention path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline and
``--impl reference`` legs may import this package. It wraps ``dd_oracle.c``
(a plain-C restatement of ReferenceBackend::decode_batch,
crates/dendrite-core/src/attention/backend.rs:206-283, of
merge_attention_outputs, crates/dendrite-ffi/src/flashinfer/cascade.rs:116-124,
and of the FP8 E4M3 / MXFP8 codec following
crates/dendrite-core/src/quantization/fp8.rs:103-152 and OCP MX v1.0).

Parity status: attention numerics "parity unpinned" — the reference has no
golden vectors for them and cannot be built here; the restatement is
cross-checked against torch CPU math. FP8 codes are pinned to ml_dtypes /
torch float8 casts via tests/golden.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _cpu_has_v3() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return all(f" {f}" in flags for f in ("avx2", "fma", "bmi2"))


def _load():
    name = "liboracle_v3.so" if _cpu_has_v3() else "liboracle_generic.so"
    path = HERE / name
    if not path.exists() or path.stat().st_mtime < (HERE / "dd_oracle.c").stat().st_mtime:
        from . import build as _b  # build recipe lives beside the source
        _b.build()
    lib = C.CDLL(str(path))
    vp, i64 = C.c_void_p, C.c_int64
    sig = {
        "or_prefill": (None, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp, vp, vp, vp]),
        "or_decode_batch": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp,
                                      C.c_int, i64, vp, vp, vp, vp, vp, vp, C.c_int]),
        "or_decode_batch_ws": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp,
                                         C.c_int, i64, vp, vp, vp, vp, vp, vp, C.c_int, vp, C.c_size_t]),
        "or_decode_scratch_floats": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
        "or_merge_states": (None, [C.c_int, C.c_int, vp, vp, vp, vp, vp, vp]),
        "or_quant_per_head": (None, [vp, C.c_int, i64, C.c_int, C.c_int, C.c_int, vp, vp]),
        "or_quant_mx": (None, [vp, C.c_int, i64, vp, vp]),
        "or_dequant": (None, [vp, C.c_int, vp, i64, C.c_int, C.c_int, vp, C.c_int]),
        "or_e4m3_encode_n": (None, [vp, i64, vp]),
        "or_e4m3_decode_n": (None, [vp, i64, vp]),
        "or_f32_to_bf16_n": (None, [vp, i64, vp]),
        "or_head_scale": (C.c_float, [C.c_float, C.c_int]),
    }
    for k, (r, a) in sig.items():
        f = getattr(lib, k)
        f.restype, f.argtypes = r, a
    return lib, name


lib, LIB_NAME = _load()


def _p(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


def f32_to_bf16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib.or_f32_to_bf16_n(_p(x), x.size, _p(out))
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib.or_e4m3_encode_n(_p(x), x.size, _p(out))
    return out


def e4m3_decode(c) -> np.ndarray:
    c = np.ascontiguousarray(c, dtype=np.uint8)
    out = np.empty(c.shape, dtype=np.float32)
    lib.or_e4m3_decode_n(_p(c), c.size, _p(out))
    return out


def head_scale(amax: float, mode: int = 0) -> float:
    return float(lib.or_head_scale(amax, mode))


def _pool_arg(pool: np.ndarray):
    if pool.dtype == np.float32:
        return pool, 2
    if pool.dtype == np.uint16:
        return pool, 1
    raise TypeError("pool must be float32 or uint16 (bf16 bits)")


def quantize_per_head(pool: np.ndarray, mode: int = 0):
    """pool [P][2][Hkv][16][D] f32 or bf16 bits -> (codes uint8, scales f32[2, Hkv])."""
    pool, dt = _pool_arg(np.ascontiguousarray(pool))
    P, _, Hkv, _, D = pool.shape
    codes = np.empty(pool.shape, dtype=np.uint8)
    scales = np.empty((2, Hkv), dtype=np.float32)
    lib.or_quant_per_head(_p(pool), dt, P, Hkv, D, mode, _p(codes), _p(scales))
    return codes, scales


def quantize_mx(pool: np.ndarray):
    """-> (codes uint8 same shape, E8M0 scales uint8 [..., D/32])."""
    pool, dt = _pool_arg(np.ascontiguousarray(pool))
    codes = np.empty(pool.shape, dtype=np.uint8)
    scales = np.empty(pool.shape[:-1] + (pool.shape[-1] // 32,), dtype=np.uint8)
    lib.or_quant_mx(_p(pool), dt, pool.size, _p(codes), _p(scales))
    return codes, scales


def dequantize(codes: np.ndarray, scales: np.ndarray, fmt: str, out: str = "bf16") -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    P, _, Hkv, _, D = codes.shape
    o = np.empty(codes.shape, dtype=np.uint16 if out == "bf16" else np.float32)
    sc = np.ascontiguousarray(scales, dtype=np.float32 if fmt == "e4m3" else np.uint8)
    lib.or_dequant(_p(codes), 3 if fmt == "e4m3" else 4, _p(sc), P, Hkv, D, _p(o),
                   1 if out == "bf16" else 2)
    return o


def prefill(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float = 0.0) -> np.ndarray:
    """ReferenceBackend::prefill (backend.rs:163-204), batch 1: q [Hq][S][D],
    k, v [Hkv][S][D] f32 -> causal attention output [Hq][S][D] f32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    Hq, S, D = q.shape
    out = np.empty((Hq, S, D), dtype=np.float32)
    lib.or_prefill(S, Hq, k.shape[0], D, scale, _p(q), _p(k), _p(v), _p(out))
    return out


class DecodeScratch:
    """Per-thread gather / repeat scratch of decode_batch, allocated and
    touched once so repeated (timed) calls do not pay for page faults."""

    def __init__(self, threads: int, Hq: int, Hkv: int, D: int, max_tokens: int):
        self.threads = int(threads)
        self.per_thread = int(lib.or_decode_scratch_floats(Hq, Hkv, D, int(max_tokens)))
        self.buf = np.ones(self.threads * self.per_thread, dtype=np.float32)


def decode_batch(q: np.ndarray, pool: np.ndarray, indptr, block_ids, num_tokens, num_kv_heads: int,
                 gqa_grouped: bool = False, scale: float = 0.0, threads: int | None = None,
                 scratch: DecodeScratch | None = None):
    """ReferenceBackend::decode_batch. q [B][Hq][D] f32; pool f32 or bf16 bits.
    Returns (out f32 [B][Hq][D], lse f32 [B][Hq] natural log). With scratch,
    its threads run the batch in its preallocated buffers."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    pool, dt = _pool_arg(np.ascontiguousarray(pool))
    B, Hq, D = q.shape
    indptr = np.ascontiguousarray(indptr, dtype=np.int32)
    ids = np.ascontiguousarray(block_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    ntok = np.ascontiguousarray(num_tokens, dtype=np.int32)
    out = np.empty((B, Hq, D), dtype=np.float32)
    lse = np.empty((B, Hq), dtype=np.float32)
    if scratch is not None:
        lib.or_decode_batch_ws(B, Hq, num_kv_heads, D, 1 if gqa_grouped else 0, scale, _p(pool), dt,
                               pool.shape[0], _p(q), _p(indptr), _p(ids), _p(ntok), _p(out),
                               _p(lse), scratch.threads, _p(scratch.buf), scratch.per_thread)
        return out, lse
    threads = threads or os.cpu_count() or 1
    lib.or_decode_batch(B, Hq, num_kv_heads, D, 1 if gqa_grouped else 0, scale, _p(pool), dt,
                        pool.shape[0], _p(q), _p(indptr), _p(ids), _p(ntok), _p(out), _p(lse),
                        int(threads))
    return out, lse


def merge_states(o1, l1, o2, l2):
    o1, o2 = (np.ascontiguousarray(a, dtype=np.float32) for a in (o1, o2))
    l1, l2 = (np.ascontiguousarray(a, dtype=np.float32) for a in (l1, l2))
    n, D = l1.size, o1.shape[-1]
    o = np.empty_like(o1)
    l = np.empty_like(l1)
    lib.or_merge_states(n, D, _p(o1), _p(l1), _p(o2), _p(l2), _p(o), _p(l))
    return o, l
