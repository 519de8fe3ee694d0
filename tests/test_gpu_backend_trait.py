"""The drop-in trait methods of B200Backend (decode, decode_batch, append_kv)
driven through the same sequences as the reference's own backend tests
(crates/dendrite-core/src/attention/backend.rs: decode with an empty cache
:417, decode with a cache :431, decode_batch of two :451, append_kv :482),
plus a multi-block copy-on-write tree, each result compared with the oracle
(ReferenceBackend::decode_batch restated in C). append_kv goes through the
C entry point dd_append_kv.

The reference's tests build their tensors with Tensor::randn and check shapes
only; here the same shapes come from a seeded generator and the values are
checked as well. Our BlockTable carries its token count (the reference's
BlockTable has the same field, block_table.rs:14): a block filled by a
16-token store is a table with num_tokens 16.
"""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import workloads as wl
from tests.helpers import F32_MAX_ABS, F32_MEAN_REL, assert_close, bf16_bits, bits_to_f32

pytestmark = pytest.mark.gpu


def _randn(g, *shape, device):
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float32)


def _oracle_one(backend, queries, tables, config, dtype):
    """Oracle over the backend's pool for queries [1, Hq, 1, D] and tables."""
    pool = backend.pages.float().cpu().numpy() if backend.pages.dtype == torch.float32 else \
        backend.pages.view(torch.int16).cpu().numpy().view(np.uint16)
    q = torch.stack([x.reshape(config.num_heads, config.head_dim) for x in queries]).float().cpu().numpy()
    indptr = np.cumsum([0] + [t.num_blocks() for t in tables]).astype(np.int32)
    ids = np.array([b for t in tables for b in t.blocks()], dtype=np.uint32)
    ntok = np.array([t.num_tokens() for t in tables], dtype=np.int32)
    ref, _ = oracle.decode_batch(q, pool, indptr, ids, ntok, config.num_kv_heads,
                                 gqa_grouped=backend.gqa_map == dd._lib.GQA_GROUPED)
    if dtype == torch.bfloat16:
        ref = bits_to_f32(bf16_bits(ref))
    return ref


def test_decode_empty_cache(cuda):
    """backend.rs:417: an empty block table decodes to zeros of the query's shape."""
    backend = dd.B200Backend(num_pages=4, num_kv_heads=4, head_dim=64, kv_dtype="f32", device=cuda)
    config = dd.AttentionConfig(4, 4, 64)
    g = torch.Generator(device=cuda).manual_seed(417)
    query = _randn(g, 1, 4, 1, 64, device=cuda)
    out = backend.decode(query, dd.BlockTable(16), config)
    torch.cuda.synchronize()
    assert out.shape == query.shape and out.dtype == query.dtype
    assert torch.all(out == 0)


def test_decode_with_cache(cuda):
    """backend.rs:431: 16 tokens stored in block 0, one query over it."""
    backend = dd.B200Backend(num_pages=4, num_kv_heads=4, head_dim=64, kv_dtype="f32", device=cuda)
    config = dd.AttentionConfig(4, 4, 64)
    g = torch.Generator(device=cuda).manual_seed(431)
    table = dd.BlockTable(16)
    table.push(0)
    backend.append_kv(_randn(g, 1, 4, 16, 64, device=cuda), _randn(g, 1, 4, 16, 64, device=cuda), table, 0)
    table.set_num_tokens(16)
    query = _randn(g, 1, 4, 1, 64, device=cuda)
    out = backend.decode(query, table, config)
    torch.cuda.synchronize()
    assert out.shape == query.shape and out.dtype == query.dtype
    ref = _oracle_one(backend, [query], [table], config, torch.float32)
    assert_close(out.reshape(1, 4, 64).cpu().numpy(), ref, F32_MAX_ABS, F32_MEAN_REL, "decode with cache")


def test_decode_batch_two(cuda):
    """backend.rs:451: blocks 0 and 1 stored, one query over each."""
    backend = dd.B200Backend(num_pages=4, num_kv_heads=4, head_dim=64, kv_dtype="f32", device=cuda)
    config = dd.AttentionConfig(4, 4, 64)
    g = torch.Generator(device=cuda).manual_seed(451)
    tables = []
    for blk in (0, 1):
        t = dd.BlockTable(16)
        t.push(blk)
        backend.append_kv(_randn(g, 1, 4, 16, 64, device=cuda), _randn(g, 1, 4, 16, 64, device=cuda), t, 0)
        t.set_num_tokens(16)
        tables.append(t)
    queries = [_randn(g, 1, 4, 1, 64, device=cuda) for _ in range(2)]
    outs = backend.decode_batch(queries, tables, config)
    torch.cuda.synchronize()
    assert len(outs) == 2
    assert all(o.shape == q.shape and o.dtype == q.dtype for o, q in zip(outs, queries))
    ref = _oracle_one(backend, queries, tables, config, torch.float32)
    got = torch.stack([o.reshape(4, 64) for o in outs]).cpu().numpy()
    assert_close(got, ref, F32_MAX_ABS, F32_MEAN_REL, "decode_batch")
    # Each batch entry equals its own decode (the batch shares no prefix here).
    for i in range(2):
        one = backend.decode(queries[i], tables[i], config)
        assert_close(one.cpu().numpy(), outs[i].cpu().numpy(), F32_MAX_ABS, F32_MEAN_REL, "decode vs batch")


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_append_kv(cuda, kv_dtype):
    """backend.rs:482 (one token at position 0 of block 0), plus tokens landing
    mid-block through the table and a position without a block (ignored, as
    the reference ignores it)."""
    backend = dd.B200Backend(num_pages=3, num_kv_heads=4, head_dim=64, kv_dtype=kv_dtype, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(482)
    table = dd.BlockTable(16)
    table.push(2)
    table.push(0)
    before = backend.pages.clone()
    k = _randn(g, 1, 4, 1, 64, device=cuda)
    v = _randn(g, 1, 4, 1, 64, device=cuda)
    backend.append_kv(k, v, table, 0)  # block 2, slot 0
    k3 = _randn(g, 1, 4, 3, 64, device=cuda)
    v3 = _randn(g, 1, 4, 3, 64, device=cuda)
    backend.append_kv(k3, v3, table, 21)  # block 0, slots 5..7
    backend.append_kv(k, v, table, 40)  # logical block 2 does not exist: ignored
    torch.cuda.synchronize()
    dt = backend.pages.dtype
    exp = before.clone()
    exp[2, 0, :, 0] = k[0, :, 0].to(dt)
    exp[2, 1, :, 0] = v[0, :, 0].to(dt)
    exp[0, 0, :, 5:8] = k3[0].to(dt)
    exp[0, 1, :, 5:8] = v3[0].to(dt)
    assert torch.equal(backend.pages, exp)


@pytest.mark.parametrize("kv_dtype,gqa", [("bf16", dd._lib.GQA_TILED), ("bf16", dd._lib.GQA_GROUPED),
                                          ("f32", dd._lib.GQA_TILED)])
def test_tree_through_the_trait(cuda, kv_dtype, gqa):
    """A copy-on-write tree (shared root, forked nodes, partial last pages)
    written token by token with append_kv and decoded with decode_batch;
    Llama-3-8B heads (32 query / 8 KV, head_dim 128)."""
    tb = wl.small_tree(13, Hq=32, Hkv=8, D=128, prefix=320, levels=((3, 16, 64),), leaves_per_node=3,
                       suffix=(1, 37))
    backend = dd.B200Backend(num_pages=tb.num_pages, num_kv_heads=8, head_dim=128, kv_dtype=kv_dtype,
                             device=cuda, gqa_map=gqa)
    config = dd.AttentionConfig(32, 8, 128)
    g = torch.Generator(device=cuda).manual_seed(13)
    tables = []
    written = set()
    for b in range(tb.batch_size):
        ids = tb.block_ids[tb.indptr[b]:tb.indptr[b + 1]].tolist()
        t = dd.BlockTable(16, ids, int(tb.num_tokens[b]))
        tables.append(t)
        # Store every page this table covers once, in 16-token (or partial) appends.
        for i, blk in enumerate(ids):
            if blk in written:
                continue
            written.add(blk)
            n = min(16, int(tb.num_tokens[b]) - 16 * i)
            if n <= 0:
                continue
            backend.append_kv(_randn(g, 1, 8, n, 128, device=cuda), _randn(g, 1, 8, n, 128, device=cuda),
                              t, 16 * i)
    qdt = torch.float32 if kv_dtype == "f32" else torch.bfloat16
    queries = [_randn(g, 1, 32, 1, 128, device=cuda).to(qdt) for _ in range(tb.batch_size)]
    outs = backend.decode_batch(queries, tables, config)
    torch.cuda.synchronize()
    got = torch.stack([o.reshape(32, 128) for o in outs]).float().cpu().numpy()
    ref = _oracle_one(backend, queries, tables, config, qdt)
    if kv_dtype == "f32":
        assert_close(got, ref, F32_MAX_ABS, F32_MEAN_REL, "f32 tree")
    else:
        assert_close(got, ref, what=f"bf16 tree gqa={gqa}")
    # decode() of one leaf equals its batch entry.
    one = backend.decode(queries[-1], tables[-1], config)
    assert_close(one.float().reshape(1, 32, 128).cpu().numpy(), got[-1:], what="decode vs batch")
