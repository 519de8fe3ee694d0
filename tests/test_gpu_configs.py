"""GPU parity on the configurations bench.py times, at their full sizes.

Each case builds its tree with bench.py's own generator and seed
(``bench.make_tree``) and its pool and queries with ``bench.device_inputs``,
runs the cascade decode the benchmark times, and compares it with the oracle
(the C restatement of ReferenceBackend::decode_batch,
crates/dendrite-core/src/attention/backend.rs:206-283) at the north_star
bounds (tests/helpers.py):

* config 3 (512-leaf Llama-3-8B MCTS tree, bf16 KV): every query;
* config 4 (config 3 over per-head E4M3 and MXFP8 pages): every query, against
  the oracle on the bit-identical dequantised pages (bf16 bounds) and against
  the bf16-KV oracle (1.25x the oracle's own FP8 error);
* config 5a (Llama-3-70B heads, 32768-token prefix + 64 x 256): one whole tree
  from the forest generator (bench.py decodes 64 of them per step at N=1);
* config 5b (one 131072-token prefix + 256 x 256): the full batch decoded on one
  GPU and through the emulated 8-way KV-head split (each rank's shard decoded
  in turn, stacked as the all-gather does, reordered by
  dd_scatter_head_shards), the oracle on a fixed subset of 16 queries;
* the tcgen05 path over FP8 pages with x50 outliers (large scale factors).

The oracle runs on the host's cores (memory-capped thread count).
"""
import numpy as np
import pytest
import torch

import bench
import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from dendrite_b200 import head_split as hs
from dendrite_b200 import workloads as wl
from tests.helpers import (FP8_MAX_ABS_CAP, FP8_MEAN_REL_CAP, assert_close, bf16_bits, bits_to_f32,
                           errors, random_pool)

pytestmark = pytest.mark.gpu

_CACHE = {}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _oracle(tb, pool_np, q_f32, n=None, gqa=0):
    """Oracle over the first n queries (all by default), rounded to bf16 as
    the reference returns the query's dtype."""
    n = tb.batch_size if n is None else n
    ip = tb.indptr[: n + 1]
    threads = bench.oracle_threads(tb)
    ref, lse = oracle.decode_batch(q_f32[:n], pool_np, ip, tb.block_ids[: ip[-1]], tb.num_tokens[:n],
                                   tb.num_kv_heads, gqa_grouped=bool(gqa), threads=threads)
    return bits_to_f32(bf16_bits(ref)), lse


def _decode(tb, cfg, q, kv, scales=None):
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
    plan.upload(q.device)
    _lib.profile_enable(True)
    out, lse = dd.cascade_decode(cfg, plan, q, kv, scales)
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    return out, lse, prof


def _config3(cuda):
    if "c3" not in _CACHE:
        tb, _ = bench.make_tree("mcts8b", 0, 1)
        pool, q = bench.device_inputs(tb, bench.pool_pages(tb), bench.SEED, cuda)
        q_f32 = q.float().cpu().numpy()
        ref, ref_lse = _oracle(tb, _bits(pool), q_f32)
        _CACHE["c3"] = (tb, pool, q, q_f32, ref, ref_lse)
    return _CACHE["c3"]


def test_config3_full(cuda):
    tb, pool, q, _, ref, ref_lse = _config3(cuda)
    assert tb.batch_size == 512
    cfg = dd.make_config(32, 8, 128, pool.shape[0])
    out, lse, prof = _decode(tb, cfg, q, pool)
    assert prof["attn_tc"][1] >= 1 and prof["attn_mma"][1] >= 1
    assert_close(out.float().cpu().numpy(), ref, what="config 3")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
def test_config4_full(cuda, fmt):
    tb, pool, q, q_f32, ref_bf16, _ = _config3(cuda)
    codes, scales = dd.quantize_kv_pages(pool, fmt)
    kvd = _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8
    cfg = dd.make_config(32, 8, 128, pool.shape[0], kv_dtype=kvd)
    out, lse, prof = _decode(tb, cfg, q, codes, scales)
    assert prof["attn_tc"][1] >= 1 and prof["attn_mma"][1] >= 1
    got = out.float().cpu().numpy()
    deq = oracle.dequantize(codes.cpu().numpy(), scales.cpu().numpy(), fmt)
    ref_fp8, ref_lse = _oracle(tb, deq, q_f32)
    assert_close(got, ref_fp8, what=f"config 4 {fmt} vs dequantised oracle")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)
    oma, omr = errors(ref_fp8, ref_bf16)
    assert oma <= FP8_MAX_ABS_CAP and omr <= FP8_MEAN_REL_CAP, (oma, omr)
    assert_close(got, ref_bf16, 1.25 * oma, 1.25 * omr, f"config 4 {fmt} vs bf16-KV oracle")


def test_config5a_one_tree(cuda):
    tb = wl.llama3_70b_forest(num_trees=1, seed=bench.SEED)
    pool, q = bench.device_inputs(tb, tb.num_pages, bench.SEED, cuda)
    cfg = dd.make_config(64, 8, 128, tb.num_pages)
    out, lse, prof = _decode(tb, cfg, q, pool)
    assert prof["attn_tc"][1] >= 1
    ref, ref_lse = _oracle(tb, _bits(pool), q.float().cpu().numpy())
    assert_close(out.float().cpu().numpy(), ref, what="config 5a, one tree")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


def test_config5b_full_and_split(cuda):
    tb, _ = bench.make_tree("long70b", 0, 1)
    assert tb.batch_size == 256
    pool, q = bench.device_inputs(tb, bench.pool_pages(tb), bench.SEED, cuda)
    cfg = dd.make_config(64, 8, 128, pool.shape[0])
    n = 16
    ref, ref_lse = _oracle(tb, _bits(pool), q.float().cpu().numpy(), n=n)
    # One GPU, all heads.
    out1, lse1, prof = _decode(tb, cfg, q, pool)
    assert prof["attn_tc"][1] >= 1
    assert_close(out1[:n].float().cpu().numpy(), ref, what="config 5b, one GPU")
    np.testing.assert_allclose(lse1[:n].cpu().numpy(), ref_lse, atol=2e-3)
    # The 8-way KV-head split, each rank's shard in turn.
    world = 8
    lcfg = hs.shard_config(cfg, world)
    shards = []
    for r in range(world):
        plan = dd.CascadePlan(lcfg, tb.indptr, tb.block_ids, tb.num_tokens)
        o, _ = dd.cascade_decode(lcfg, plan, hs.shard_queries(q, cfg, r, world),
                                 hs.shard_pages(pool, r, world))
        shards.append(o)
    gathered = torch.stack(shards).contiguous()
    out8 = torch.empty_like(q)
    dd.scatter_head_shards(cfg, world, gathered, out8)
    torch.cuda.synchronize()
    assert_close(out8[:n].float().cpu().numpy(), ref, what="config 5b, 8-way split")
    # Every query of the split agrees with the unsplit decode.
    assert_close(out8.float().cpu().numpy(), out1.float().cpu().numpy(), what="split vs one GPU")


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
def test_fp8_tcgen05_with_outliers(cuda, fmt):
    """A wide shared root (64 leaves x 4 GQA rows = 256 rows: the tcgen05
    kernel) over FP8 pages quantised from values with 0.1% x50 outliers, so
    the per-head scales and MX exponents are far from 1. Against the oracle on
    the dequantised pages: mean-rel 1e-3, and max-abs 2e-2 or one bf16 ulp of
    the largest output, whichever is larger (outputs reach ~50, where one
    bf16 ulp is 0.25)."""
    tb = wl.build_tree("fp8outliers", 32, 8, 128, 2048, [(4, 64, 256)], 16, (1, 100), 77)
    rng = np.random.default_rng(77)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128, outliers=1e-3))
    qb = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    to_dev = lambda b: torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16).to(cuda)  # noqa: E731
    codes, scales = dd.quantize_kv_pages(to_dev(pool), fmt)
    kvd = _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8
    cfg = dd.make_config(32, 8, 128, tb.num_pages, kv_dtype=kvd)
    out, _, prof = _decode(tb, cfg, to_dev(qb), codes, scales)
    assert prof["attn_tc"][1] >= 1
    deq = oracle.dequantize(codes.cpu().numpy(), scales.cpu().numpy(), fmt)
    ref, _ = _oracle(tb, deq, bits_to_f32(qb))
    top = float(np.abs(ref).max())
    ulp = 2.0 ** (np.floor(np.log2(top)) - 7) if top > 0 else 0.0
    assert_close(out.float().cpu().numpy(), ref, max(2e-2, ulp), what=f"{fmt} outliers")
