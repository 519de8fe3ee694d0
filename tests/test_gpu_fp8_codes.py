"""Exactness of the FP8 -> bf16 widening inside the attention kernels.

A query that sees a single token gets that token's V row back (softmax weight
exactly 1), so the output equals the dequantised V codes. The V rows here
enumerate all 256 E4M3 codes (NaNs and subnormals included) and MXFP8
exponent bytes from 0 to 255 (246 is the largest whose products stay
finite: an infinite V element meets the zero low half of the split softmax
weight and gives NaN where the f32 reference gives inf), and the result must match the oracle's
dequantisation bit for bit (NaN where it has NaN) through both the tcgen05
kernel (32 queries share the page: 128 rows) and the streaming kernel."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from tests.helpers import bf16_bits, bits_to_f32

pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 128


def _pool(fmt, rng):
    P = 2
    codes = rng.integers(0, 0x7e, size=(P, 2, HKV, 16, D), dtype=np.uint8)  # finite K/V
    codes[..., :] |= (rng.integers(0, 2, size=codes.shape, dtype=np.uint8) << 7)
    v0 = np.tile(np.arange(256, dtype=np.uint8), (HKV * D) // 256).reshape(HKV, D)
    codes[0, 1, :, 0, :] = v0  # V of token 0, page 0: every code 4 times
    if fmt == "e4m3":
        scales = np.array([[0.37, 1.0, 2.5e-3, 7.0, 0.011, 1.5, 0.5, 3.0],
                           [1.0, 0.37, 2.5e-3, 9.0, 0.013, 1.25, 0.75, 1e-5]], np.float32)
    else:
        scales = rng.integers(120, 131, size=(P, 2, HKV, 16, D // 32), dtype=np.uint8)
        scales[0, 1, :, 0, :] = np.array([[127, 0, 134, 135], [140, 255, 1, 100],
                                          [126, 128, 133, 136], [50, 90, 200, 246],
                                          [127, 127, 127, 127], [3, 7, 131, 132],
                                          [110, 120, 125, 129], [60, 70, 80, 137]], np.uint8)
    return codes, scales


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
@pytest.mark.parametrize("tc", [True, False])
def test_single_token_returns_dequantised_v(cuda, fmt, tc):
    rng = np.random.default_rng(17)
    codes, scales = _pool(fmt, rng)
    nq = 32
    indptr = np.arange(nq + 1, dtype=np.int32)
    ids = np.zeros(nq, np.uint32)
    ntok = np.ones(nq, np.int32)
    q = bf16_bits(rng.standard_normal((nq, HQ, D)).astype(np.float32))
    kvd = _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8
    cfg = dd.make_config(HQ, HKV, D, codes.shape[0], kv_dtype=kvd)
    plan = dd.CascadePlan(cfg, indptr, ids, ntok, use_tensor_cores=tc)
    plan.upload(cuda)
    qd = torch.from_numpy(q.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    _lib.profile_enable(True)
    out, _ = dd.cascade_decode(cfg, plan, qd, torch.from_numpy(codes).to(cuda),
                               torch.from_numpy(scales).to(cuda))
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    assert (prof["attn_tc"][1] >= 1) == tc, prof
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    deq = oracle.dequantize(codes, scales, fmt, out="f32")
    ref, _ = oracle.decode_batch(bits_to_f32(q), deq, indptr, ids, ntok, HKV)
    want = bf16_bits(ref)
    # query head h reads KV head h % 8 (tiled GQA); every query sees token 0
    exp_v = bf16_bits(deq[0, 1, np.arange(HQ) % HKV, 0, :])
    nan_g, nan_w = np.isnan(bits_to_f32(got)), np.isnan(bits_to_f32(want))
    assert np.array_equal(nan_g, nan_w)
    assert np.array_equal(np.where(nan_w, 0, got), np.where(nan_w, 0, want))
    # (values, not bits: the oracle's 1 * (-0) accumulates to +0)
    np.testing.assert_array_equal(bits_to_f32(want[0]), bits_to_f32(exp_v))
