"""Pins the CPU oracle to the golden fixtures (no GPU)."""
import numpy as np
import pytest

import oracle
from tests.helpers import bits_to_f32


def test_e4m3_decode_all_codes(golden):
    g = golden["fp8_codec"]["e4m3_decode"]
    got = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))
    nan = np.isnan(g)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan], g[~nan])
    assert nan.sum() == 2  # 0x7F and 0xFF


def test_e4m3_encode_kat(golden):
    g = golden["fp8_codec"]
    got = oracle.e4m3_encode(g["enc_x"])
    bad = np.nonzero(got != g["enc_code"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={g['enc_x'][bad[:5]]}"


def test_e4m3_encode_roundtrip_every_code():
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], dtype=np.uint8)
    back = oracle.e4m3_encode(oracle.e4m3_decode(codes))
    # -0 encodes to 0x80, +0 to 0x00; everything else round-trips exactly.
    assert np.array_equal(back, codes)


def test_e4m3_saturates_like_reference_clamp():
    # fp8.rs:130 clamps t/scale to +-448 before storing.
    x = np.array([448, 449, 464, 1e30, np.inf, -500, -np.inf], dtype=np.float32)
    assert list(oracle.e4m3_encode(x)) == [0x7E, 0x7E, 0x7E, 0x7E, 0x7E, 0xFE, 0xFE]


def test_e8m0_decode(golden):
    g = golden["fp8_codec"]["e8m0_decode"]
    # Decode through the MX dequantiser: code 0x38 (1.0) times 2^(s-127).
    codes = np.full((256, 2, 1, 16, 32), 0x38, dtype=np.uint8)
    scales = np.repeat(np.arange(256, dtype=np.uint8), 2 * 16).reshape(256, 2, 1, 16, 1)
    got = oracle.dequantize(codes, scales, "mxfp8", out="f32")[:, 0, 0, 0, 0]
    ok = ~np.isnan(g)
    assert np.array_equal(got[ok], g[ok])
    assert np.isnan(got[255])


def test_per_head_quant_kat(golden):
    g = golden["quant_kv"]
    codes, scales = oracle.quantize_per_head(g["pool_bf16_bits"], mode=0)
    assert np.array_equal(scales, g["head_scales"])
    assert np.array_equal(codes, g["head_codes"])
    deq = oracle.dequantize(codes, scales, "e4m3", out="bf16")
    assert np.array_equal(deq, g["head_deq_bf16_bits"])


def test_mx_quant_kat(golden):
    g = golden["quant_kv"]
    codes, scales = oracle.quantize_mx(g["pool_bf16_bits"])
    assert np.array_equal(scales, g["mx_scales"])
    assert np.array_equal(codes, g["mx_codes"])
    deq = oracle.dequantize(codes, scales, "mxfp8", out="bf16")
    assert np.array_equal(deq, g["mx_deq_bf16_bits"])


def test_mx_zero_and_tiny_blocks():
    x = np.zeros((1, 2, 1, 16, 64), dtype=np.float32)
    x[0, 0, 0, 0, 32:64] = 1e-40  # subnormal block: e clamps at -127
    codes, scales = oracle.quantize_mx(x)
    assert scales[0, 0, 0, 0, 0] == 0 and np.all(codes[0, 0, 0, 0, :32] == 0)
    assert scales[0, 0, 0, 0, 1] == 0
    assert np.all(codes[0, 0, 0, 0, 32:] == oracle.e4m3_encode(np.float32(1e-40) * np.float32(2.0 ** 127)))


def test_head_scale_modes():
    # mode 0: amax * f32(1/448) (candle affine); mode 1: amax / 448; zero -> 1.
    a = np.float32(3.7)
    assert oracle.head_scale(float(a), 0) == float(a * np.float32(1.0 / 448.0))
    assert oracle.head_scale(float(a), 1) == float(a / np.float32(448.0))
    assert oracle.head_scale(0.0, 0) == 1.0


def test_attention_oracle_matches_f64(golden):
    g = golden["attention_small"]
    out, lse = oracle.decode_batch(g["q"], g["pool"], g["indptr"], g["block_ids"],
                                   g["num_tokens"], int(g["num_kv_heads"]), threads=2)
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=0)
    fin = np.isfinite(g["lse"])
    np.testing.assert_allclose(lse[fin], g["lse"][fin], atol=2e-5)
    assert np.all(out[3] == 0) and np.all(np.isneginf(lse[3]))  # empty table -> zeros


def test_attention_oracle_bf16_pool_equals_f32_of_rounded(golden):
    g = golden["attention_small"]
    bits = oracle.f32_to_bf16_bits(g["pool"])
    a, _ = oracle.decode_batch(g["q"], bits, g["indptr"], g["block_ids"], g["num_tokens"], 2)
    b, _ = oracle.decode_batch(g["q"], bits_to_f32(bits), g["indptr"], g["block_ids"],
                               g["num_tokens"], 2)
    assert np.array_equal(a, b)


def test_grouped_gqa_differs_from_tiled(golden):
    g = golden["attention_small"]
    a, _ = oracle.decode_batch(g["q"], g["pool"], g["indptr"], g["block_ids"], g["num_tokens"], 2)
    b, _ = oracle.decode_batch(g["q"], g["pool"], g["indptr"], g["block_ids"], g["num_tokens"], 2,
                               gqa_grouped=True)
    assert np.array_equal(a[:, 0], b[:, 0])       # head 0 reads KV head 0 either way
    assert not np.allclose(a[:, 1], b[:, 1])      # head 1: KV 1 (tiled) vs KV 0 (grouped)


@pytest.mark.parametrize("seed", [0, 1])
def test_merge_states_formula(seed):
    rng = np.random.default_rng(seed)
    o1, o2 = rng.standard_normal((2, 7, 16)).astype(np.float32)
    l1, l2 = (rng.standard_normal((2, 7)) * 5).astype(np.float32)
    o, l = oracle.merge_states(o1, l1, o2, l2)
    m = np.maximum(l1, l2)
    e1, e2 = np.exp(l1 - m), np.exp(l2 - m)
    np.testing.assert_allclose(o, (o1 * e1[:, None] + o2 * e2[:, None]) / (e1 + e2)[:, None],
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l, m + np.log(e1 + e2), rtol=1e-6, atol=1e-6)
