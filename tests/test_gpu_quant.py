"""GPU KV-page quantize / dequantize against the oracle, bit for bit.

Config 2: a pool of 4096 pages x [2 (K,V)][4 KV heads][16 tokens][64 dims]
bf16 (33.5 M elements, 67.1 MB), N(0,1) with 0.1% of the elements x50.
Codes and scales must equal the oracle's exactly for per-head E4M3 (both
scale modes) and MXFP8, and the bf16 / f32 round trip must equal the
oracle's dequantisation. Edge pages: an all-zero head (scale 1 / exponent
code 0), values past the E4M3 range (saturate to +-448), tiny values
(subnormal codes), mixed signs of zero."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from tests.helpers import bf16_bits, random_pool

pytestmark = pytest.mark.gpu


def _pool(P=4096, Hkv=4, D=64, seed=2):
    rng = np.random.default_rng(seed)
    x = random_pool(rng, P, Hkv, D, outliers=1e-3)
    x[0, :, 0] = 0.0                        # all-zero page/head slice
    x[1, 0, 1, :, :] = 3.0e4                 # far past 448 * scale for most blocks
    x[1, 1, 1, :, :8] = -1.0e-30             # tiny values: subnormal codes / zeros
    x[2, 0, 2, 3, :] = -0.0
    return bf16_bits(x)


def _dev(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("fmt,mode", [("e4m3", 0), ("e4m3", 1), ("mxfp8", 0)])
def test_quantize_config2_bit_exact(cuda, fmt, mode):
    bits = _pool()
    codes, scales = dd.quantize_kv_pages(_dev(bits, cuda), fmt, scale_mode=mode)
    torch.cuda.synchronize()
    if fmt == "e4m3":
        oc, os_ = oracle.quantize_per_head(bits, mode=mode)
    else:
        oc, os_ = oracle.quantize_mx(bits)
    got_c, got_s = codes.cpu().numpy(), scales.cpu().numpy()
    assert np.array_equal(got_s.view(np.uint8), os_.view(np.uint8)), "scales differ"
    bad = np.nonzero(got_c != oc)
    assert bad[0].size == 0, f"{bad[0].size} codes differ, first at {[b[0] for b in bad]}"
    for out_dtype, name in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
        deq = dd.dequantize_kv_pages(codes, scales, fmt, out_dtype=out_dtype)
        torch.cuda.synchronize()
        want = oracle.dequantize(oc, os_, fmt, out=name)
        got = deq.view(torch.int16).cpu().numpy().view(np.uint16) if name == "bf16" else deq.cpu().numpy()
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), f"{name} round trip differs"


def test_quantize_f32_source_matches_oracle(cuda):
    x = oracle.bf16_bits_to_f32(_pool(P=64))
    x = x * np.float32(1.0 + 1e-3)           # values that are not bf16-representable
    for fmt in ("e4m3", "mxfp8"):
        codes, scales = dd.quantize_kv_pages(torch.from_numpy(x).to(cuda), fmt)
        torch.cuda.synchronize()
        oc, os_ = oracle.quantize_per_head(x) if fmt == "e4m3" else oracle.quantize_mx(x)
        assert np.array_equal(codes.cpu().numpy(), oc)
        assert np.array_equal(scales.cpu().numpy().view(np.uint8), os_.view(np.uint8))
