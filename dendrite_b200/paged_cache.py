"""Paged KV cache for a model's decode loop: the attention step of
TransformerLayer::forward_with_cache
(crates/dendrite-core/src/model/layer.rs:374-416) over a page pool per layer
instead of the contiguous LayerCache, with one cascade plan per step for all
layers.

forward_with_cache appends the step's RoPE'd K/V to the layer's cache
(`cache.append`, :392-393) and attends with `compute_attention` (:276-318):
scale 1/sqrt(head_dim), GQA by `repeat_kv` (:321-340), an unsqueeze-expand-
reshape that gives query head h the KV head h // (Hq / Hkv) (the grouped
map). Here a step of B sequences (the leaves of a tree) is:

* ``begin_step(tables, positions)``: the sequences' block tables (CSR) and
  the position of each one's new token. The plan is advanced in place when
  every sequence only grew by that token (``CascadePlan.advance``, a new block
  read from its table when the token starts one) and re-planned otherwise
  (first step, a fork, a copy-on-write); it is uploaded once for all layers.
* ``layer_step(layer, q, k, v)``: stores the new token's K/V of that layer
  into its pool at (table[pos // 16], pos % 16) — quantised for FP8 pools —
  and runs the cascade decode of q [B, Hq, D] over the pool with the shared
  plan; returns the attention output [B, Hq, D] (what compute_attention
  returns before the output projection).

Prompts go in through ``layer_prefill`` (the causal prefill plan of the new
tokens over their sequence, ReferenceBackend::prefill's attention when the
sequence starts empty).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .backend import (PAGE_SIZE, CascadePlan, _alloc_ws, append_kv_batch, cascade_decode,
                      make_config)

_KV = {"bf16": _lib.DTYPE_BF16, "e4m3": _lib.DTYPE_E4M3, "mxfp8": _lib.DTYPE_MXFP8}


class PagedKVCache:
    """Page pools of `num_layers` layers ([num_pages][2][Hkv][16][D] each) and
    the step's cascade plan, shared by the layers."""

    def __init__(self, num_layers: int, num_pages: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, kv_dtype: str = "bf16", e4m3_scales=None,
                 device: str | torch.device = "cuda"):
        if kv_dtype not in _KV:
            raise _lib.InvalidArgument("kv_dtype must be bf16, e4m3 or mxfp8")
        self.device = torch.device(device)
        self.Hq, self.Hkv, self.D, self.num_pages = num_heads, num_kv_heads, head_dim, num_pages
        self.kv_dtype = kv_dtype
        self.cfg = make_config(num_heads, num_kv_heads, head_dim, num_pages, kv_dtype=_KV[kv_dtype],
                               gqa_map=_lib.GQA_GROUPED)
        shape = (num_pages, 2, num_kv_heads, PAGE_SIZE, head_dim)
        if kv_dtype == "bf16":
            self.pools = [torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
                          for _ in range(num_layers)]
            self.scales = [None] * num_layers
        else:
            self.pools = [torch.zeros(shape, dtype=torch.uint8, device=self.device)
                          for _ in range(num_layers)]
            if kv_dtype == "mxfp8":
                self.scales = [torch.zeros(shape[:-1] + (head_dim // 32,), dtype=torch.uint8,
                                           device=self.device) for _ in range(num_layers)]
            else:
                if e4m3_scales is None:
                    raise _lib.InvalidArgument("per-head E4M3 pages need e4m3_scales ([2][Hkv] per layer)")
                self.scales = [torch.as_tensor(s, dtype=torch.float32).reshape(2, num_kv_heads)
                               .contiguous().to(self.device) for s in e4m3_scales]
        self.plan: CascadePlan | None = None
        self._ntok = None
        self._tables = None
        self._ws: dict = {}
        self._page_ids = self._slots = None

    # -- per step ---------------------------------------------------------
    def _only_grew(self, indptr, block_ids) -> bool:
        """Every table is the previous step's, with at most one block appended."""
        pi, pb = self._tables
        old_len, new_len = np.diff(pi), np.diff(indptr)
        if len(old_len) != len(new_len) or np.any((new_len < old_len) | (new_len > old_len + 1)):
            return False
        idx = np.repeat(indptr[:-1], old_len) + (np.arange(int(pi[-1])) - np.repeat(pi[:-1], old_len))
        return bool(np.array_equal(block_ids[idx], pb[:int(pi[-1])]))

    def begin_step(self, indptr, block_ids, positions, tree_grew_only: bool | None = None) -> bool:
        """Plan the step. positions[b]: the new token's index in sequence b
        (so it holds positions[b] + 1 tokens after the step). The plan is
        advanced in place when every sequence only gained this token (and
        maybe a block for it) since the last step — checked against the
        previous tables unless the caller says so with tree_grew_only=True —
        and re-planned otherwise. Returns True when advanced."""
        indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        block_ids = np.ascontiguousarray(block_ids, dtype=np.uint32)
        pos = np.ascontiguousarray(positions, dtype=np.int64)
        ntok = (pos + 1).astype(np.int32)
        blk = block_ids[indptr[:-1] + pos // PAGE_SIZE]
        advanced = False
        if self.plan is not None and self._ntok is not None and len(self._ntok) == len(ntok) \
                and np.array_equal(self._ntok + 1, ntok) \
                and (tree_grew_only or (tree_grew_only is None and self._only_grew(indptr, block_ids))):
            advanced = self.plan.advance(np.ones(len(ntok), np.int32), blk)
        if not advanced:
            if self.plan is None:
                self.plan = CascadePlan(self.cfg, indptr, block_ids, ntok)
            else:
                self.plan.rebuild(indptr, block_ids, ntok)
        self.plan.upload(self.device)
        self._ntok = ntok
        self._tables = (indptr.copy(), block_ids.copy())
        self._page_ids = torch.from_numpy(blk.astype(np.int32)).to(self.device)
        self._slots = torch.from_numpy((pos % PAGE_SIZE).astype(np.int32)).to(self.device)
        return advanced

    def layer_step(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Store layer `layer`'s new K/V [B, Hkv, D] and attend with q [B, Hq, D]."""
        append_kv_batch(self.cfg, self.pools[layer], self.scales[layer], self._page_ids, self._slots,
                        k.contiguous(), v.contiguous())
        q = q.to(torch.bfloat16).contiguous()
        ws = _alloc_ws(self.plan.info().workspace_bytes, self.device, self._ws)
        out, _ = cascade_decode(self.cfg, self.plan, q, self.pools[layer], self.scales[layer],
                                workspace=ws)
        return out

    # -- prompts ------------------------------------------------------------
    def layer_prefill(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      table, prefix_len: int) -> torch.Tensor:
        """One sequence's S new tokens: store their K/V [S, Hkv, D] at
        positions prefix_len .. prefix_len + S of `table` and return the
        causal attention of q [S, Hq, D] (new token i sees tokens
        0 .. prefix_len + i)."""
        S = q.shape[0]
        pos = np.arange(prefix_len, prefix_len + S)
        tbl = np.asarray(table, dtype=np.uint32)
        page_ids = torch.from_numpy(tbl[pos // PAGE_SIZE].astype(np.int32)).to(self.device)
        slots = torch.from_numpy((pos % PAGE_SIZE).astype(np.int32)).to(self.device)
        append_kv_batch(self.cfg, self.pools[layer], self.scales[layer], page_ids, slots,
                        k.contiguous(), v.contiguous())
        plan = CascadePlan.prefill(self.cfg, [0, len(tbl)], tbl, [prefix_len], [S])
        plan.upload(self.device)
        out, _ = cascade_decode(self.cfg, plan, q.to(torch.bfloat16).contiguous(), self.pools[layer],
                                self.scales[layer])
        return out
