"""GPU parity of the tcgen05 kernel (wide shared nodes) against the oracle."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from dendrite_b200 import workloads as wl
from tests.helpers import assert_close, bf16_bits, bits_to_f32, random_pool

pytestmark = pytest.mark.gpu


def _dev_bf16(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _run(tb, pool_bits, q_bits, dev, tc=True, gqa=0, pairs=False):
    cfg = dd.make_config(tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.num_pages, gqa_map=gqa)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, use_tensor_cores=tc,
                          cta_pairs=pairs)
    plan.upload(dev)
    launches = _lib.launch_count()
    _lib.profile_enable(True)
    out, lse = dd.cascade_decode(cfg, plan, _dev_bf16(q_bits, dev), _dev_bf16(pool_bits, dev))
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    return out.float().cpu().numpy(), lse.cpu().numpy(), prof, _lib.launch_count() - launches


def _groups(groups, seed):
    """Queries in groups sharing one whole table each: [(n_queries, tokens)]."""
    rng = np.random.default_rng(seed)
    ids, indptr, ntok, nxt = [], [0], [], 0
    for nq, tok in groups:
        nb = -(-tok // 16)
        tab = list(range(nxt, nxt + nb))
        nxt += nb
        for _ in range(nq):
            ids += tab
            indptr.append(len(ids))
            ntok.append(tok)
    perm = rng.permutation(nxt).astype(np.uint32)
    return np.array(indptr, np.int32), perm[np.array(ids, np.int64)], np.array(ntok, np.int32), nxt


class _TB:
    def __init__(self, Hq, Hkv, D, indptr, ids, ntok, P):
        self.num_qo_heads, self.num_kv_heads, self.head_dim = Hq, Hkv, D
        self.indptr, self.block_ids, self.num_tokens, self.num_pages = indptr, ids, ntok, P
        self.batch_size = len(ntok)


CASES = [
    # (Hq, Hkv, prefix, leaves, suffix range, gqa)
    (32, 8, 1008, 37, (1, 40), 0),     # 148 root rows: tiles of 128 + 20; 63 pages
    (32, 8, 2048, 64, (16, 200), 1),   # grouped GQA, 256 rows
    (64, 8, 4096, 64, (1, 300), 0),    # g = 8, 512 rows, 32 token tiles
    (32, 4, 496, 40, (1, 17), 0),      # 320 rows over 31 pages (one partial tile)
]


@pytest.mark.parametrize("pairs", [False, True])
@pytest.mark.parametrize("Hq,Hkv,prefix,leaves,suffix,gqa", CASES)
def test_wide_root_vs_oracle(cuda, Hq, Hkv, prefix, leaves, suffix, gqa, pairs):
    """pairs: nodes of > 256 rows on the CTA-pair (cta_group::2) kernel."""
    seed = Hq + prefix + leaves
    tb = wl.build_tree("wide", Hq, Hkv, 128, prefix, [], leaves, suffix, seed)
    rng = np.random.default_rng(seed)
    pool = bf16_bits(random_pool(rng, tb.num_pages, Hkv, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, Hq, 128)).astype(np.float32))
    got, lse, prof, _ = _run(tb, pool, q, cuda, gqa=gqa, pairs=pairs)
    assert prof["attn_tc"][1] >= 1, prof  # the wide root went through tcgen05
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), pool, tb.indptr, tb.block_ids,
                                       tb.num_tokens, Hkv, gqa_grouped=bool(gqa))
    assert_close(got, bits_to_f32(bf16_bits(ref)), what="tc root")
    np.testing.assert_allclose(lse, ref_lse, atol=2e-3)


def test_shared_partial_last_page_through_tc(cuda):
    indptr, ids, ntok, P = _groups([(40, 1000), (1, 37), (33, 129)], 3)
    tb = _TB(32, 8, 128, indptr, ids, ntok, P)
    rng = np.random.default_rng(3)
    pool = bf16_bits(random_pool(rng, P, 8, 128))
    q = bf16_bits(rng.standard_normal((len(ntok), 32, 128)).astype(np.float32))
    got, lse, prof, _ = _run(tb, pool, q, cuda)
    assert prof["attn_tc"][1] >= 1
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), pool, indptr, ids, ntok, 8)
    assert_close(got, bits_to_f32(bf16_bits(ref)), what="partial pages")
    np.testing.assert_allclose(lse, ref_lse, atol=2e-3)


def test_tc_matches_mma_path(cuda):
    tb = wl.build_tree("cmp", 32, 8, 128, 3072, [(4, 128, 512)], 16, (1, 100), 9)
    rng = np.random.default_rng(9)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    a, la, pa, _ = _run(tb, pool, q, cuda, tc=True)
    b, lb, pb, _ = _run(tb, pool, q, cuda, tc=False)
    assert pa["attn_tc"][1] >= 1 and pb["attn_tc"][1] == 0
    assert_close(a, b, what="tc vs mma")
    np.testing.assert_allclose(la, lb, atol=1e-3)


def test_large_score_range_rescales(cuda):
    """Keys whose scores grow along the sequence force the lazy O rescale."""
    indptr, ids, ntok, P = _groups([(48, 2048)], 4)
    tb = _TB(32, 8, 128, indptr, ids, ntok, P)
    rng = np.random.default_rng(4)
    x = random_pool(rng, P, 8, 128)
    # page order along the sequence gets a growing key scale: scores climb by
    # far more than 2^8 across tiles
    order = ids[:ntok[0] // 16 + 1]
    for i, p in enumerate(order):
        x[p, 0] *= 1.0 + 0.15 * i
    pool = bf16_bits(x)
    q = bf16_bits(rng.standard_normal((len(ntok), 32, 128)).astype(np.float32))
    got, lse, prof, _ = _run(tb, pool, q, cuda)
    assert prof["attn_tc"][1] >= 1
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), pool, indptr, ids, ntok, 8)
    assert_close(got, bits_to_f32(bf16_bits(ref)), what="rescale")
    np.testing.assert_allclose(lse, ref_lse, rtol=1e-4, atol=1e-2)


def test_score_jump_inside_a_tile(cuda):
    """A page of very large keys in the second 64-token chunk of the first
    tile and another in a later tile: the single-pass softmax moves its
    reference mid-tile and rescales the P it already wrote, O and the sum."""
    indptr, ids, ntok, P = _groups([(40, 1024)], 6)
    tb = _TB(32, 8, 128, indptr, ids, ntok, P)
    rng = np.random.default_rng(6)
    x = random_pool(rng, P, 8, 128)
    order = ids[:ntok[0] // 16]
    x[order[5], 0] *= 40.0    # tile 0, chunk 1 (tokens 80-95)
    x[order[37], 0] *= 80.0   # tile 4
    pool = bf16_bits(x)
    q = bf16_bits(rng.standard_normal((len(ntok), 32, 128)).astype(np.float32))
    got, lse, prof, _ = _run(tb, pool, q, cuda)
    assert prof["attn_tc"][1] >= 1
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), pool, indptr, ids, ntok, 8)
    assert_close(got, bits_to_f32(bf16_bits(ref)), what="score jump")
    np.testing.assert_allclose(lse, ref_lse, rtol=1e-4, atol=1e-2)


@pytest.mark.parametrize("pairs", [False, True])
def test_mcts_subset_vs_oracle(cuda, pairs):
    """A 128-leaf version of the MCTS tree (root through tcgen05), all queries."""
    tb = wl.build_tree("mcts128", 32, 8, 128, 8192, [(4, 128, 1024), (4, 128, 1024), (2, 128, 1024)],
                       4, (16, 256), 0xD3D1)
    rng = np.random.default_rng(1)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    got, lse, prof, n = _run(tb, pool, q, cuda, pairs=pairs)
    assert prof["attn_tc"][1] >= 1 and n >= 3
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), pool, tb.indptr, tb.block_ids, tb.num_tokens, 8)
    assert_close(got, bits_to_f32(bf16_bits(ref)), what="mcts128")
    np.testing.assert_allclose(lse, ref_lse, atol=2e-3)


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
@pytest.mark.parametrize("prefix,gqa", [(1008, 0), (2050, 1)])
def test_fp8_wide_root_vs_oracle(cuda, fmt, prefix, gqa):
    """FP8 pages through tcgen05: codes widened to bf16 in shared memory (exact
    for E4M3; per-head scales applied to S and O, MXFP8 exponents per element).
    Compared with the oracle over the f32 dequantised pool at the bf16 bounds.
    1008 tokens leave the last tile with one absent page; 2050 a 2-token page."""
    tb = wl.build_tree("fp8wide", 32, 8, 128, prefix, [], 40, (1, 40), prefix)
    rng = np.random.default_rng(prefix)
    # No outliers here: x50 values make outputs of ~100, where one bf16 ulp
    # (0.5) exceeds the absolute bound; the outlier case is covered by the
    # FP8 tree test.
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    codes, scales = dd.quantize_kv_pages(_dev_bf16(pool, cuda), fmt)
    kvd = _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8
    cfg = dd.make_config(32, 8, 128, tb.num_pages, kv_dtype=kvd, gqa_map=gqa)
    outs = {}
    for tc in (True, False):
        plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, use_tensor_cores=tc)
        plan.upload(cuda)
        _lib.profile_enable(True)
        out, lse = dd.cascade_decode(cfg, plan, _dev_bf16(q, cuda), codes, scales)
        torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
        assert (prof["attn_tc"][1] >= 1) == tc, prof
        outs[tc] = (out.float().cpu().numpy(), lse.cpu().numpy())
    deq = oracle.dequantize(codes.cpu().numpy(), scales.cpu().numpy(), fmt)
    ref, ref_lse = oracle.decode_batch(bits_to_f32(q), deq, tb.indptr, tb.block_ids, tb.num_tokens, 8,
                                       gqa_grouped=bool(gqa))
    assert_close(outs[True][0], bits_to_f32(bf16_bits(ref)), what=f"{fmt} tc")
    np.testing.assert_allclose(outs[True][1], ref_lse, atol=2e-3)
    assert_close(outs[True][0], outs[False][0], what=f"{fmt} tc vs mma")
