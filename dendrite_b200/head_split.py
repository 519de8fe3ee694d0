"""KV-head split of one long tree across GPUs (one process per GPU).

A tree too long for one GPU's time budget is split by KV-head group, not by
sequence: rank r of W owns KV heads [r*Hkv/W, (r+1)*Hkv/W) of every page and
the query heads that read them under the GQA map, decodes them with the
ordinary cascade plan (the plan depends only on the block tables, so every
rank builds the same one), and the per-rank outputs [B][Hq/W][D] are joined
by one all-gather over NVLink plus a reorder kernel (dd_scatter_head_shards).
No partial states cross GPUs: each query head is computed whole on one rank.

Local head numbering follows the GQA map restricted to the rank's KV heads,
so the local problem is itself a valid (Hq/W, Hkv/W) configuration:

* tiled (``h % Hkv``, ReferenceBackend's ``Tensor::repeat``,
  crates/dendrite-core/src/attention/backend.rs:245-252): local head
  ``j*c + i`` (c = Hkv/W) is global head ``k0 + i + j*Hkv``;
* grouped (``h / g``, crates/dendrite-core/src/model/layer.rs:321-340): local
  head ``i*g + j`` is global head ``(k0 + i)*g + j``.
"""
from __future__ import annotations

import torch

from . import _lib
from .backend import AttnConfig, CascadePlan, cascade_decode, make_config, scatter_head_shards  # noqa: F401


def kv_heads_of(rank: int, world: int, num_kv_heads: int) -> range:
    """KV heads owned by `rank`."""
    if world <= 0 or num_kv_heads % world:
        raise _lib.InvalidArgument(f"num_kv_heads {num_kv_heads} does not split over {world} ranks")
    c = num_kv_heads // world
    return range(rank * c, (rank + 1) * c)


def query_heads_of(rank: int, world: int, num_qo_heads: int, num_kv_heads: int,
                   gqa_map: int = _lib.GQA_TILED) -> list[int]:
    """Global query heads of `rank`, in local head order."""
    ks = kv_heads_of(rank, world, num_kv_heads)
    g = num_qo_heads // num_kv_heads
    if gqa_map == _lib.GQA_TILED:
        return [k + j * num_kv_heads for j in range(g) for k in ks]
    return [k * g + j for k in ks for j in range(g)]


def shard_config(cfg: AttnConfig, world: int) -> AttnConfig:
    """The rank-local configuration: Hq/W query heads over Hkv/W KV heads,
    same head_dim, page count, dtypes, GQA map and softmax scale."""
    if cfg.num_kv_heads % world or cfg.num_qo_heads % world:
        raise _lib.InvalidArgument("head counts do not split over the world size")
    return make_config(cfg.num_qo_heads // world, cfg.num_kv_heads // world, cfg.head_dim,
                       cfg.num_pages, kv_dtype=cfg.kv_dtype, q_dtype=cfg.q_dtype,
                       gqa_map=cfg.gqa_map, scale=cfg.scale)


def shard_pages(pages: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's KV heads of a page pool [P][2][Hkv][16][D] (codes included)."""
    ks = kv_heads_of(rank, world, pages.shape[2])
    return pages[:, :, ks.start:ks.stop].contiguous()


def shard_scales(scales: torch.Tensor | None, kv_dtype: int, rank: int, world: int,
                 num_kv_heads: int) -> torch.Tensor | None:
    """This rank's FP8 scales: per-head E4M3 f32[2][Hkv], or MXFP8 E8M0
    [P][2][Hkv][16][D/32]."""
    if scales is None:
        return None
    ks = kv_heads_of(rank, world, num_kv_heads)
    if kv_dtype == _lib.DTYPE_E4M3:
        return scales.reshape(2, num_kv_heads)[:, ks.start:ks.stop].contiguous()
    return scales[:, :, ks.start:ks.stop].contiguous()


def shard_queries(q: torch.Tensor, cfg: AttnConfig, rank: int, world: int) -> torch.Tensor:
    """This rank's query heads of q [B][Hq][D], in local order."""
    heads = query_heads_of(rank, world, cfg.num_qo_heads, cfg.num_kv_heads, cfg.gqa_map)
    return q[:, heads].contiguous()


def head_split_decode(cfg: AttnConfig, plan_local: CascadePlan, q_local: torch.Tensor,
                      kv_local: torch.Tensor, scales_local: torch.Tensor | None,
                      world: int, group=None, out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode this rank's head shard, all-gather the shards, reorder to
    out [B][Hq][D]. `plan_local` is a plan made with shard_config(cfg, world);
    the collective is torch.distributed's all_gather_into_tensor on `group`
    (NCCL over NVLink on a GPU box)."""
    import torch.distributed as dist

    lcfg = shard_config(cfg, world)
    local_out, _ = cascade_decode(lcfg, plan_local, q_local, kv_local, scales_local, workspace=workspace)
    B = q_local.shape[0]
    gathered = torch.empty((world,) + tuple(local_out.shape), dtype=local_out.dtype,
                           device=local_out.device)
    if world > 1:
        dist.all_gather_into_tensor(gathered, local_out, group=group)
    else:
        gathered[0].copy_(local_out)
    if out is None:
        out = torch.empty((B, cfg.num_qo_heads, cfg.head_dim), dtype=local_out.dtype,
                          device=local_out.device)
    return scatter_head_shards(cfg, world, gathered, out)


def allgather_heads(nccl_comm: int, cfg: AttnConfig, world: int, local_out: torch.Tensor,
                    out: torch.Tensor | None = None, gathered: torch.Tensor | None = None,
                    stream=None) -> torch.Tensor:
    """dd_allgather_heads: the same join through the C ABI, on a raw
    ncclComm_t (an integer handle) owned by the caller."""
    import ctypes as C

    from .backend import _ptr, _stream

    B = local_out.shape[0]
    if gathered is None:
        gathered = torch.empty((world,) + tuple(local_out.shape), dtype=local_out.dtype,
                               device=local_out.device)
    if out is None:
        out = torch.empty((B, cfg.num_qo_heads, cfg.head_dim), dtype=local_out.dtype,
                          device=local_out.device)
    _lib.check(_lib.lib.dd_allgather_heads(C.c_void_p(nccl_comm), C.byref(cfg), world, B,
                                           _ptr(local_out), _ptr(gathered), _ptr(out),
                                           _stream(stream)), "dd_allgather_heads")
    return out



class FusedHeadSplit:
    """The head split with the join fused into the decode
    (dd_cascade_decode_shards): the final merge of every rank writes its rows
    straight into all ranks' output buffers over NVLink, so no all-gather and
    no reorder kernel run. The outputs live in symmetric memory (torch's
    CUDA-backend allocation, mapped into every rank), two buffers used in
    turn; after each decode the ranks meet at a device-side barrier, so the
    returned buffer is complete, and a buffer is written again only after
    every rank has passed the next step's barrier (by then each rank has
    consumed it in stream order)."""

    def __init__(self, cfg: AttnConfig, world: int, rank: int, batch_size: int, device,
                 group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.cfg, self.world, self.rank = cfg, world, rank
        self.lcfg = shard_config(cfg, world)
        if symm.get_backend(device) is None:
            symm.set_backend("CUDA")
        g = group if group is not None else dist.group.WORLD
        dtype = torch.bfloat16 if cfg.q_dtype == _lib.DTYPE_BF16 else torch.float32
        self.bufs, self.handles = [], []
        for _ in range(2):
            t = symm.empty((batch_size, cfg.num_qo_heads, cfg.head_dim), dtype=dtype, device=device)
            self.bufs.append(t)
            self.handles.append(symm.rendezvous(t, g))
        self.step = 0

    def decode(self, plan_local: CascadePlan, q_local: torch.Tensor, kv_local: torch.Tensor,
               scales_local: torch.Tensor | None, lse_local: torch.Tensor,
               workspace: torch.Tensor, stream=None) -> torch.Tensor:
        import ctypes as C

        from .backend import _ptr, _stream

        i = self.step % 2
        h = self.handles[i]
        if plan_local.device_buffer is None:
            plan_local.upload(q_local.device, stream)
        _lib.check(_lib.lib.dd_cascade_decode_shards(
            C.byref(self.lcfg), plan_local._h, _ptr(q_local), _ptr(kv_local), _ptr(scales_local),
            C.c_void_p(int(h.buffer_ptrs_dev)), self.world, self.rank, self.cfg.num_qo_heads,
            self.cfg.num_kv_heads, _ptr(lse_local), _ptr(workspace), workspace.numel(),
            _stream(stream)), "dd_cascade_decode_shards")
        h.barrier(channel=0)
        self.step += 1
        return self.bufs[i]
