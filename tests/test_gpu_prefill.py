"""GPU causal prefill over pages (dd_plan_create_prefill + dd_cascade_decode)
against the oracle: the restatement of ReferenceBackend::prefill
(crates/dendrite-core/src/attention/backend.rs:163-204) for sequences without
a prefix, and the decode restatement over nested token counts (query i of a
sequence sees its first prefix + i + 1 tokens) otherwise."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from tests.helpers import (F32_MAX_ABS, F32_MEAN_REL, assert_close, bf16_bits, bits_to_f32,
                           random_pool)

pytestmark = pytest.mark.gpu


def _bf16_dev(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _tables(rng, P, prefix, new):
    perm = rng.permutation(P)
    indptr, ids, off = [0], [], 0
    for p_, n_ in zip(prefix, new):
        k = (p_ + n_ + 15) // 16
        ids += list(perm[off:off + k])
        off += k
        indptr.append(len(ids))
    return np.array(indptr, np.int32), np.array(ids, np.uint32)


def _nested_oracle(q_f32, pool, indptr, ids, prefix, new, Hkv):
    qi_ptr, qi_ids, qi_ntok = [0], [], []
    for s, (p_, n_) in enumerate(zip(prefix, new)):
        tbl = ids[indptr[s]:indptr[s + 1]]
        for i in range(n_):
            qi_ids += list(tbl)
            qi_ptr.append(len(qi_ids))
            qi_ntok.append(p_ + i + 1)
    return oracle.decode_batch(q_f32, pool, np.array(qi_ptr, np.int32), np.array(qi_ids, np.uint32),
                               np.array(qi_ntok, np.int32), Hkv)


def _run(cfg, dev, indptr, ids, prefix, new, q_dev, pool_dev, scales=None):
    plan = dd.CascadePlan.prefill(cfg, indptr, ids, prefix, new)
    plan.upload(dev)
    out, lse = dd.cascade_decode(cfg, plan, q_dev, pool_dev, scales)
    torch.cuda.synchronize()
    return out, lse, plan


@pytest.mark.parametrize("Hq,Hkv,prefix,new", [
    (8, 8, [0], [37]),                       # 37 rows: streaming kernel
    (32, 8, [300], [100]),                   # 400 rows: tcgen05 row tiles, pages trimmed per tile
    (32, 8, [0, 45, 1000], [20, 70, 33]),    # three sequences, both kernels
    (8, 2, [16], [1]),                       # one new token = a decode step
])
def test_prefill_bf16_vs_oracle(cuda, Hq, Hkv, prefix, new):
    rng = np.random.default_rng(sum(prefix) + 7 * sum(new))
    D, P = 128, 160
    indptr, ids = _tables(rng, P, prefix, new)
    pool = bf16_bits(random_pool(rng, P, Hkv, D))
    T = sum(new)
    q = bf16_bits(rng.standard_normal((T, Hq, D)).astype(np.float32))
    cfg = dd.make_config(Hq, Hkv, D, P)
    out, lse, _ = _run(cfg, cuda, indptr, ids, prefix, new, _bf16_dev(q, cuda), _bf16_dev(pool, cuda))
    ref, ref_lse = _nested_oracle(bits_to_f32(q), pool, indptr, ids, prefix, new, Hkv)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what=f"prefill {prefix}/{new}")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


def test_prefill_branches_share_prefix(cuda):
    """Chunked prefill of branch suffixes over one shared prefix: a 300-token
    prefix (18 full pages shared, its partial page copied per branch, as
    copy-on-write does), then each branch's own new tokens."""
    rng = np.random.default_rng(21)
    Hq, Hkv, D, P = 32, 8, 128, 128
    prefix, new = 300, [33, 7, 80, 1, 45, 16]
    perm = rng.permutation(P)
    shared, nxt = list(perm[:19]), 19
    pool = random_pool(rng, P, Hkv, D)
    tables = []
    for n_ in new:
        own = list(perm[nxt:nxt + (prefix + n_ + 15) // 16 - 18])
        nxt += len(own)
        pool[own[0], :, :, :prefix % 16] = pool[shared[18], :, :, :prefix % 16]  # copy-on-write
        tables.append(shared[:18] + own)
    indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    ids = np.concatenate(tables).astype(np.uint32)
    pool = bf16_bits(pool)
    q = bf16_bits(rng.standard_normal((sum(new), Hq, D)).astype(np.float32))
    cfg = dd.make_config(Hq, Hkv, D, P)
    out, _, plan = _run(cfg, cuda, indptr, ids, [prefix] * len(new), new, _bf16_dev(q, cuda),
                        _bf16_dev(pool, cuda))
    n = plan.nodes()
    assert n["num_q"][n["parent"] < 0].max() == sum(new)    # the shared pages: one node for all
    ref, _ = _nested_oracle(bits_to_f32(q), pool, indptr, ids, [prefix] * len(new), new, Hkv)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="branch prefill")


def test_prefill_f32_tinyllama_shapes(cuda):
    """f32 pages (CUDA-core kernel), TinyLlama heads, against the restatement
    of ReferenceBackend::prefill itself (no prefix)."""
    rng = np.random.default_rng(3)
    Hq, Hkv, D, S, P = 32, 4, 64, 45, 16
    k = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    v = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    q = rng.standard_normal((Hq, S, D)).astype(np.float32)
    ids = rng.permutation(P)[:(S + 15) // 16].astype(np.uint32)
    pool = np.zeros((P, 2, Hkv, 16, D), np.float32)
    for t in range(S):
        pool[ids[t // 16], 0, :, t % 16] = k[:, t]
        pool[ids[t // 16], 1, :, t % 16] = v[:, t]
    cfg = dd.make_config(Hq, Hkv, D, P, kv_dtype=_lib.DTYPE_F32, q_dtype=_lib.DTYPE_F32)
    out, _, _ = _run(cfg, cuda, [0, len(ids)], ids, [0], [S],
                     torch.from_numpy(q.transpose(1, 0, 2).copy()).to(cuda), torch.from_numpy(pool).to(cuda))
    ref = oracle.prefill(q, k, v)
    assert_close(out.cpu().numpy().transpose(1, 0, 2), ref, F32_MAX_ABS, F32_MEAN_REL, "prefill f32")


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
def test_prefill_fp8_vs_dequantised_oracle(cuda, fmt):
    rng = np.random.default_rng(11)
    Hq, Hkv, D, P = 32, 8, 128, 96
    prefix, new = [200, 3], [64, 150]
    indptr, ids = _tables(rng, P, prefix, new)
    pool = bf16_bits(random_pool(rng, P, Hkv, D))
    q = bf16_bits(rng.standard_normal((sum(new), Hq, D)).astype(np.float32))
    codes, scales = dd.quantize_kv_pages(_bf16_dev(pool, cuda), fmt)
    kvd = _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8
    cfg = dd.make_config(Hq, Hkv, D, P, kv_dtype=kvd)
    out, _, _ = _run(cfg, cuda, indptr, ids, prefix, new, _bf16_dev(q, cuda), codes, scales)
    deq = oracle.dequantize(codes.cpu().numpy(), scales.cpu().numpy(), fmt, out="bf16")
    ref, _ = _nested_oracle(bits_to_f32(q), deq, indptr, ids, prefix, new, Hkv)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what=f"prefill {fmt}")


def test_backend_prefill_matches_reference_prefill(cuda):
    """B200Backend.prefill (trait method, backend.rs:163-204): stores the new
    tokens' K/V in the block table's pages and returns the reference's dense
    causal attention; a later decode sees the stored tokens."""
    rng = np.random.default_rng(9)
    Hq, Hkv, D, S = 8, 2, 128, 40
    be = dd.B200Backend(num_pages=32, num_kv_heads=Hkv, head_dim=D, device=cuda)
    cfg = dd.AttentionConfig(num_heads=Hq, num_kv_heads=Hkv, head_dim=D)
    bt = dd.BlockTable(blocks=[5, 9, 2], num_tokens=S)
    qb = bf16_bits(rng.standard_normal((1, Hq, S, D)).astype(np.float32))
    kb = bf16_bits(rng.standard_normal((1, Hkv, S, D)).astype(np.float32))
    vb = bf16_bits(rng.standard_normal((1, Hkv, S, D)).astype(np.float32))
    out = be.prefill(_bf16_dev(qb, cuda), _bf16_dev(kb, cuda), _bf16_dev(vb, cuda), bt, cfg)
    assert out.shape == (1, Hq, S, D)
    ref = oracle.prefill(bits_to_f32(qb)[0], bits_to_f32(kb)[0], bits_to_f32(vb)[0])
    assert_close(out.float().cpu().numpy()[0], bits_to_f32(bf16_bits(ref)), what="backend prefill")
    # the K/V landed in the pages: decoding the last query token again matches
    q_last = _bf16_dev(qb, cuda)[:, :, S - 1:S, :]
    dec = be.decode(q_last, bt, cfg)
    assert_close(dec.float().cpu().numpy()[0, :, 0], out.float().cpu().numpy()[0, :, S - 1],
                 what="decode after prefill")
