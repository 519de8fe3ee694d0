"""Host logic of the KV-head split (one long tree over W ranks), run as two
gloo ranks on CPU: each rank takes its KV heads of the pool and its query
heads (dendrite_b200.head_split), computes them with the oracle, the ranks
all-gather, and the reorder must rebuild exactly the full-head result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dendrite_b200 import _lib
from dendrite_b200 import head_split as hs
from dendrite_b200 import workloads as wl


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(Hq, Hkv, gqa):
    import oracle
    from tests.helpers import bf16_bits, random_pool

    tb = wl.small_tree(21, Hq=Hq, Hkv=Hkv, D=64, prefix=300, levels=((3, 16, 64),),
                       leaves_per_node=2, suffix=(1, 30))
    rng = np.random.default_rng(21)
    pool = oracle.bf16_bits_to_f32(bf16_bits(random_pool(rng, tb.num_pages, Hkv, 64)))
    q = oracle.bf16_bits_to_f32(bf16_bits(rng.standard_normal((tb.batch_size, Hq, 64)).astype(np.float32)))
    return tb, pool, q


def _rank(rank, world, port, Hq, Hkv, gqa, result):
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tb, pool, q = _problem(Hq, Hkv, gqa)
        cfg = hs.make_config(Hq, Hkv, 64, tb.num_pages, gqa_map=gqa)
        lcfg = hs.shard_config(cfg, world)
        pool_l = hs.shard_pages(torch.from_numpy(pool), rank, world).numpy()
        q_l = hs.shard_queries(torch.from_numpy(q), cfg, rank, world).numpy()
        assert pool_l.shape[2] == lcfg.num_kv_heads and q_l.shape[1] == lcfg.num_qo_heads
        out_l, _ = oracle.decode_batch(q_l, pool_l, tb.indptr, tb.block_ids, tb.num_tokens,
                                       lcfg.num_kv_heads, gqa_grouped=bool(gqa))
        parts = [torch.empty_like(torch.from_numpy(out_l)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(out_l))
        out = np.empty((tb.batch_size, Hq, 64), np.float32)
        for r in range(world):
            out[:, hs.query_heads_of(r, world, Hq, Hkv, gqa)] = parts[r].numpy()
        full, _ = oracle.decode_batch(q, pool, tb.indptr, tb.block_ids, tb.num_tokens, Hkv,
                                      gqa_grouped=bool(gqa))
        result[rank] = float(np.abs(out - full).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("gqa", [_lib.GQA_TILED, _lib.GQA_GROUPED])
def test_head_split_two_gloo_ranks(gqa):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank, args=(r, world, port, 16, 4, gqa, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    # every query head is computed whole on one rank: bit-identical to the full run
    assert result[0] == 0.0 and result[1] == 0.0


def test_head_maps_partition_all_heads():
    for gqa in (_lib.GQA_TILED, _lib.GQA_GROUPED):
        for world in (1, 2, 4, 8):
            heads = [h for r in range(world) for h in hs.query_heads_of(r, world, 64, 8, gqa)]
            assert sorted(heads) == list(range(64))
            for r in range(world):
                ks = set(hs.kv_heads_of(r, world, 8))
                for h in hs.query_heads_of(r, world, 64, 8, gqa):
                    assert (h % 8 if gqa == _lib.GQA_TILED else h // 8) in ks
    with pytest.raises(_lib.InvalidArgument):
        hs.kv_heads_of(0, 3, 8)
