"""GPU parity of the KV-head split (one long tree over W GPUs).

* W = 2 and 4 emulated on one GPU: every rank's shard decoded in turn, the
  shards stacked as an all-gather would, reordered by dd_scatter_head_shards,
  and compared with the oracle over all heads.
* dd_allgather_heads through a one-rank NCCL communicator on one GPU.
* dd_cascade_decode_shards (the join fused into the merge) with W = 1, 2, 4
  emulated on one GPU.
* With two or more GPUs, two processes (one per GPU) join their shards with
  dd_allgather_heads over NCCL, with head_split_decode over
  torch.distributed, and with FusedHeadSplit (NVLink stores into symmetric
  memory); all must match the oracle.
"""
import ctypes as C
import os
import tempfile
import time

import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from dendrite_b200 import head_split as hs
from dendrite_b200 import workloads as wl
from tests.helpers import assert_close, bf16_bits, bits_to_f32, random_pool

pytestmark = pytest.mark.gpu

HQ, HKV, D = 64, 8, 128


def _problem(gqa, seed=31):
    tb = wl.build_tree("split", HQ, HKV, D, 4096, [], 24, (1, 200), seed)
    rng = np.random.default_rng(seed)
    pool = bf16_bits(random_pool(rng, tb.num_pages, HKV, D))
    q = bf16_bits(rng.standard_normal((tb.batch_size, HQ, D)).astype(np.float32))
    ref, _ = oracle.decode_batch(bits_to_f32(q), pool, tb.indptr, tb.block_ids, tb.num_tokens, HKV,
                                 gqa_grouped=bool(gqa))
    return tb, pool, q, bits_to_f32(bf16_bits(ref))


def _dev(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _shard_out(tb, cfg, pool_d, q_d, rank, world, dev):
    lcfg = hs.shard_config(cfg, world)
    plan = dd.CascadePlan(lcfg, tb.indptr, tb.block_ids, tb.num_tokens)
    out, _ = dd.cascade_decode(lcfg, plan, hs.shard_queries(q_d, cfg, rank, world),
                               hs.shard_pages(pool_d, rank, world))
    return out


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("gqa", [_lib.GQA_TILED, _lib.GQA_GROUPED])
def test_emulated_split_vs_oracle(cuda, world, gqa):
    tb, pool, q, ref = _problem(gqa)
    cfg = dd.make_config(HQ, HKV, D, tb.num_pages, gqa_map=gqa)
    pool_d, q_d = _dev(pool, cuda), _dev(q, cuda)
    gathered = torch.stack([_shard_out(tb, cfg, pool_d, q_d, r, world, cuda) for r in range(world)])
    out = torch.empty_like(q_d)
    dd.scatter_head_shards(cfg, world, gathered.contiguous(), out)
    torch.cuda.synchronize()
    assert_close(out.float().cpu().numpy(), ref, what=f"split x{world}")


def _shards_call(tb, cfg, pool_d, q_d, rank, world, outs, dev):
    """dd_cascade_decode_shards of one rank, writing into every buffer of `outs`."""
    from dendrite_b200.backend import _ptr

    lcfg = hs.shard_config(cfg, world)
    plan = dd.CascadePlan(lcfg, tb.indptr, tb.block_ids, tb.num_tokens)
    plan.upload(dev)
    ws = torch.empty(max(int(plan.info().workspace_bytes), 256), dtype=torch.uint8, device=dev)
    lse = torch.empty(tb.batch_size, HQ // world, dtype=torch.float32, device=dev)
    ptrs = torch.tensor([o.data_ptr() for o in outs], dtype=torch.int64, device=dev)
    _lib.check(_lib.lib.dd_cascade_decode_shards(
        C.byref(lcfg), plan._h, _ptr(hs.shard_queries(q_d, cfg, rank, world)),
        _ptr(hs.shard_pages(pool_d, rank, world)), None, C.c_void_p(ptrs.data_ptr()), world, rank,
        HQ, HKV, _ptr(lse), _ptr(ws), ws.numel(), None), "dd_cascade_decode_shards")
    torch.cuda.synchronize()


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("gqa", [_lib.GQA_TILED, _lib.GQA_GROUPED])
def test_shards_entry_emulated(cuda, world, gqa):
    """dd_cascade_decode_shards with W ranks emulated on one GPU: each rank's
    merge writes its rows into all W output buffers (here all local), which
    must each end up equal to the reordered all-gather result, and the oracle."""
    tb, pool, q, ref = _problem(gqa)
    cfg = dd.make_config(HQ, HKV, D, tb.num_pages, gqa_map=gqa)
    pool_d, q_d = _dev(pool, cuda), _dev(q, cuda)
    outs = [torch.full_like(q_d, float("nan")) for _ in range(world)]
    for r in range(world):
        _shards_call(tb, cfg, pool_d, q_d, r, world, outs, cuda)
    gathered = torch.stack([_shard_out(tb, cfg, pool_d, q_d, r, world, cuda) for r in range(world)])
    want = torch.empty_like(q_d)
    dd.scatter_head_shards(cfg, world, gathered.contiguous(), want)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)
    assert_close(outs[0].float().cpu().numpy(), ref, what=f"shards x{world}")


def _nccl():
    return C.CDLL("libnccl.so.2")


def test_allgather_heads_one_rank(cuda):
    tb, pool, q, ref = _problem(_lib.GQA_TILED)
    cfg = dd.make_config(HQ, HKV, D, tb.num_pages)
    local = _shard_out(tb, cfg, _dev(pool, cuda), _dev(q, cuda), 0, 1, cuda)
    nccl = _nccl()
    comm = C.c_void_p()
    assert nccl.ncclCommInitAll(C.byref(comm), 1, (C.c_int * 1)(cuda.index or 0)) == 0
    try:
        out = hs.allgather_heads(comm.value, cfg, 1, local)
        torch.cuda.synchronize()
    finally:
        nccl.ncclCommDestroy(comm)
    assert torch.equal(out, local)
    assert_close(out.float().cpu().numpy(), ref, what="allgather x1")


class _UniqueId(C.Structure):
    _fields_ = [("internal", C.c_byte * 128)]


def _two_gpu_rank(rank, world, idfile, port, result):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    nccl = _nccl()
    uid = _UniqueId()
    if rank == 0:
        assert nccl.ncclGetUniqueId(C.byref(uid)) == 0
        with open(idfile + ".tmp", "wb") as f:
            f.write(bytes(uid.internal))
        os.replace(idfile + ".tmp", idfile)
    else:
        for _ in range(600):
            if os.path.exists(idfile):
                break
            time.sleep(0.1)
        C.memmove(C.addressof(uid), open(idfile, "rb").read(), 128)
    comm = C.c_void_p()
    assert nccl.ncclCommInitRank(C.byref(comm), world, uid, rank) == 0
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        for gqa in (_lib.GQA_TILED, _lib.GQA_GROUPED):
            tb, pool, q, ref = _problem(gqa)
            cfg = dd.make_config(HQ, HKV, D, tb.num_pages, gqa_map=gqa)
            pool_d, q_d = _dev(pool, dev), _dev(q, dev)
            local = _shard_out(tb, cfg, pool_d, q_d, rank, world, dev)
            a = hs.allgather_heads(comm.value, cfg, world, local)
            lcfg = hs.shard_config(cfg, world)
            plan = dd.CascadePlan(lcfg, tb.indptr, tb.block_ids, tb.num_tokens)
            b = hs.head_split_decode(cfg, plan, hs.shard_queries(q_d, cfg, rank, world),
                                     hs.shard_pages(pool_d, rank, world), None, world)
            torch.cuda.synchronize()
            # The fused join: every rank's merge writes into both ranks'
            # symmetric-memory outputs; three steps (both buffers, reused).
            fh = hs.FusedHeadSplit(cfg, world, rank, tb.batch_size, dev)
            ws = torch.empty(max(int(plan.info().workspace_bytes), 256), dtype=torch.uint8, device=dev)
            lse = torch.empty(tb.batch_size, HQ // world, dtype=torch.float32, device=dev)
            for _ in range(3):
                c = fh.decode(plan, hs.shard_queries(q_d, cfg, rank, world),
                              hs.shard_pages(pool_d, rank, world), None, lse, ws)
                torch.cuda.synchronize()
                assert torch.equal(c, b)
            assert torch.equal(a, b)
            assert_close(a.float().cpu().numpy(), ref, what=f"2 GPUs gqa={gqa}")
        result[rank] = "ok"
    finally:
        dist.destroy_process_group()
        nccl.ncclCommDestroy(comm)


def test_two_gpus_allgather(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    with tempfile.TemporaryDirectory() as d:
        idfile = os.path.join(d, "nccl_id")
        procs = [ctx.Process(target=_two_gpu_rank, args=(r, 2, idfile, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
    assert all(p.exitcode == 0 for p in procs) and dict(result) == {0: "ok", 1: "ok"}
