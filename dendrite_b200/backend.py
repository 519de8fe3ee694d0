"""Host-side mirror of Dendrite's attention-backend interface over the C ABI.

``B200Backend`` implements the methods of ``trait AttentionBackend``
(crates/dendrite-core/src/attention/backend.rs:61-97) — ``decode``,
``decode_batch``, ``append_kv`` — with the same argument meaning and shapes
as ``ReferenceBackend`` (backend.rs:161-302):

* queries are ``[1, num_heads, 1, head_dim]`` tensors, outputs the same shape
  and dtype (backend.rs:212, 262);
* ``append_kv(key, value, block_table, position)`` stores ``[1, Hkv, t, D]``
  tokens in block ``block_table[position // 16]`` (backend.rs:285-301), here at
  token slots ``position % 16 ..`` of that page;
* an empty block table yields zeros (backend.rs:218-222).

KV lives in a device page pool ``[num_pages][2][Hkv][16][D]`` (the layout of
``Page``, crates/dendrite-core/src/cache/paged.rs:57). ``decode_batch`` builds
a cascade plan from the batch's block tables, so every shared prefix is read
once per batch. ``prefill`` (backend.rs:163-204) is the same causal attention
over pages: it stores the new tokens' K/V in the block table's pages and runs
a causal plan (``CascadePlan.prefill``) in which new token i sees the
sequence's tokens up to its own position.

PyTorch is used only for device memory and the current CUDA stream; all
arithmetic runs in the CUDA kernels of ``libdendrite_b200.so``.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import (DTYPE_BF16, DTYPE_E4M3, DTYPE_F32, DTYPE_MXFP8, GQA_GROUPED, GQA_TILED,
                   AttnConfig, NotAvailable, PlanInfo, PlanOptions, QuantConfig, check, lib)

PAGE_SIZE = 16                 # flashinfer/mod.rs:14
MAX_SEQ_LEN = None             # no compile-time cap (flashinfer/mod.rs:17 capped at 131072)
SUPPORTED_HEAD_DIMS = (64, 128, 256)  # flashinfer/mod.rs:20

_KV_DTYPES = {"f32": DTYPE_F32, "bf16": DTYPE_BF16, "e4m3": DTYPE_E4M3, "mxfp8": DTYPE_MXFP8}


@dataclass
class AttentionConfig:
    """Mirror of AttentionConfig (backend.rs:17-58)."""

    num_heads: int
    num_kv_heads: int
    head_dim: int
    scale: float | None = None
    sliding_window: int | None = None

    def __post_init__(self):
        if self.scale is None:
            # f32 1/sqrt(D), as backend.rs:37 computes it.
            self.scale = float(np.float32(1.0) / np.sqrt(np.float32(self.head_dim)))

    def num_queries_per_kv(self) -> int:
        return self.num_heads // self.num_kv_heads


class BlockTable:
    """Mirror of BlockTable (crates/dendrite-core/src/cache/block_table.rs:10-110)."""

    def __init__(self, tokens_per_block: int = PAGE_SIZE, blocks=None, num_tokens: int = 0):
        self.tokens_per_block = tokens_per_block
        self._blocks = list(blocks or [])
        self._num_tokens = num_tokens

    def blocks(self) -> list[int]:
        return self._blocks

    def num_blocks(self) -> int:
        return len(self._blocks)

    def num_tokens(self) -> int:
        return self._num_tokens

    def get(self, i: int):
        return self._blocks[i] if 0 <= i < len(self._blocks) else None

    def push(self, block_id: int) -> None:
        self._blocks.append(int(block_id))

    def set_num_tokens(self, n: int) -> None:
        self._num_tokens = n

    def add_tokens(self, n: int) -> None:
        self._num_tokens += n

    def needs_new_block(self) -> bool:
        if not self._blocks:
            return True
        return self._num_tokens % self.tokens_per_block == 0 and self._num_tokens > 0

    def fork(self) -> "BlockTable":
        return BlockTable(self.tokens_per_block, list(self._blocks), self._num_tokens)


def make_config(num_qo_heads: int, num_kv_heads: int, head_dim: int, num_pages: int,
                kv_dtype: int = DTYPE_BF16, q_dtype: int = DTYPE_BF16, gqa_map: int = GQA_TILED,
                scale: float = 0.0) -> AttnConfig:
    return AttnConfig(num_qo_heads, num_kv_heads, head_dim, PAGE_SIZE, kv_dtype, q_dtype, gqa_map,
                      num_pages, scale)


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class CascadePlan:
    """A prefix/suffix cascade plan built from a decode batch's block tables
    (the batch builder's output; see dd_plan_create)."""

    def __init__(self, cfg: AttnConfig, indptr, block_ids, num_tokens, share_prefixes: bool = True,
                 max_chunk_pages: int = 0, use_tensor_cores: bool = True, cta_pairs: bool = False,
                 tc_sms: int = 0):
        self.cfg = cfg
        self._indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        self._ids = np.ascontiguousarray(block_ids, dtype=np.uint32)
        self._ntok = np.ascontiguousarray(num_tokens, dtype=np.int32)
        self.batch_size = len(self._ntok)
        opts = PlanOptions(1 if share_prefixes else 0, max_chunk_pages, 1 if use_tensor_cores else 0,
                           1 if cta_pairs else 0, tc_sms)
        h = C.c_void_p()
        rc = lib.dd_plan_create(C.byref(cfg), self.batch_size,
                                self._indptr.ctypes.data_as(_lib._I32P),
                                self._ids.ctypes.data_as(_lib._U32P) if len(self._ids) else None,
                                self._ntok.ctypes.data_as(_lib._I32P), C.byref(opts), C.byref(h))
        check(rc, "dd_plan_create")
        self._h = h
        self.device_buffer = None

    @classmethod
    def prefill(cls, cfg: AttnConfig, indptr, block_ids, prefix_len, num_new,
                use_tensor_cores: bool = True) -> "CascadePlan":
        """Causal prefill plan (dd_plan_create_prefill): sequence s's last
        num_new[s] tokens are queries seeing tokens [0, prefix_len[s] + i];
        queries are numbered sequence-major."""
        self = cls.__new__(cls)
        self.cfg = cfg
        self._indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        self._ids = np.ascontiguousarray(block_ids, dtype=np.uint32)
        self._prefix = np.ascontiguousarray(prefix_len, dtype=np.int32)
        self._new = np.ascontiguousarray(num_new, dtype=np.int32)
        self._ntok = self._prefix + self._new
        self.batch_size = int(self._new.sum())
        opts = PlanOptions(1, 0, 1 if use_tensor_cores else 0, 0, 0)
        h = C.c_void_p()
        rc = lib.dd_plan_create_prefill(C.byref(cfg), len(self._new),
                                        self._indptr.ctypes.data_as(_lib._I32P),
                                        self._ids.ctypes.data_as(_lib._U32P) if len(self._ids) else None,
                                        self._prefix.ctypes.data_as(_lib._I32P),
                                        self._new.ctypes.data_as(_lib._I32P), C.byref(opts), C.byref(h))
        check(rc, "dd_plan_create_prefill")
        self._h = h
        self.device_buffer = None
        return self

    @classmethod
    def from_tables(cls, cfg: AttnConfig, tables, **kw) -> "CascadePlan":
        indptr = np.zeros(len(tables) + 1, dtype=np.int32)
        for i, t in enumerate(tables):
            indptr[i + 1] = indptr[i] + t.num_blocks()
        ids = np.array([b for t in tables for b in t.blocks()], dtype=np.uint32)
        ntok = np.array([t.num_tokens() for t in tables], dtype=np.int32)
        return cls(cfg, indptr, ids, ntok, **kw)

    def rebuild(self, indptr, block_ids, num_tokens) -> "CascadePlan":
        """Re-plan for a new batch in place (dd_plan_rebuild); the device
        buffer is kept and must be uploaded again."""
        self._indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        self._ids = np.ascontiguousarray(block_ids, dtype=np.uint32)
        self._ntok = np.ascontiguousarray(num_tokens, dtype=np.int32)
        self.batch_size = len(self._ntok)
        rc = lib.dd_plan_rebuild(self._h, self.batch_size, self._indptr.ctypes.data_as(_lib._I32P),
                                 self._ids.ctypes.data_as(_lib._U32P) if len(self._ids) else None,
                                 self._ntok.ctypes.data_as(_lib._I32P))
        check(rc, "dd_plan_rebuild")
        return self

    def advance(self, tokens_added, new_block=None) -> bool:
        """One decode step in place (dd_plan_advance): query b gained
        tokens_added[b] (0 or 1) tokens, a token that starts a new block went
        to new_block[b]. False: some query shares its last pages (or the plan
        is a prefill / flat plan); re-plan with rebuild()."""
        t = np.ascontiguousarray(tokens_added, dtype=np.int32)
        nb = None if new_block is None else np.ascontiguousarray(new_block, dtype=np.uint32)
        rc = lib.dd_plan_advance(self._h, t.ctypes.data_as(_lib._I32P),
                                 nb.ctypes.data_as(_lib._U32P) if nb is not None else None)
        if rc == _lib.DD_ERR_NOT_AVAILABLE:
            return False
        check(rc, "dd_plan_advance")
        return True

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib.dd_plan_destroy(h)
            self._h = None

    def info(self) -> PlanInfo:
        info = PlanInfo()
        check(lib.dd_plan_get_info(self._h, C.byref(info)), "dd_plan_get_info")
        return info

    def nodes(self) -> dict:
        """Host view of the plan's nodes (parent, query range, pages)."""
        info = self.info()
        n = info.num_nodes
        arrs = {k: np.zeros(n, dtype=np.int32) for k in
                ("parent", "q_begin", "num_q", "num_tokens", "page_offset", "page_count")}
        qorder = np.zeros(self.batch_size, dtype=np.int32)
        p = lambda a: a.ctypes.data_as(_lib._I32P)  # noqa: E731
        check(lib.dd_plan_export_nodes(self._h, p(arrs["parent"]), p(arrs["q_begin"]),
                                       p(arrs["num_q"]), p(arrs["num_tokens"]),
                                       p(arrs["page_offset"]), p(arrs["page_count"]), None,
                                       p(qorder)), "dd_plan_export_nodes")
        total = int(arrs["page_count"].sum()) if n else 0
        pages = np.zeros(max(total, 1), dtype=np.uint32)
        check(lib.dd_plan_export_nodes(self._h, None, None, None, None, None, None,
                                       pages.ctypes.data_as(_lib._U32P), None), "export pages")
        arrs["pages"] = pages[:total]
        arrs["query_order"] = qorder
        return arrs

    def upload(self, device=None, stream=None) -> None:
        info = self.info()
        nbytes = max(int(info.device_bytes), 256)
        if self.device_buffer is None or self.device_buffer.numel() < nbytes:
            self.device_buffer = torch.empty(nbytes, dtype=torch.uint8, device=device or "cuda")
        check(lib.dd_plan_upload(self._h, _ptr(self.device_buffer), self.device_buffer.numel(),
                                 _stream(stream)), "dd_plan_upload")


def _alloc_ws(nbytes: int, device, cache: dict | None = None, key="ws"):
    nbytes = max(int(nbytes), 256)
    if cache is not None:
        t = cache.get(key)
        if t is not None and t.numel() >= nbytes and t.device == torch.device(device):
            return t
    t = torch.empty(nbytes, dtype=torch.uint8, device=device)
    if cache is not None:
        cache[key] = t
    return t


def cascade_decode(cfg: AttnConfig, plan: CascadePlan, q: torch.Tensor, kv_pages: torch.Tensor,
                   kv_scales: torch.Tensor | None = None, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                   stream=None):
    """Cascade decode of q [B, Hq, D] over the plan. Returns (out, lse)."""
    if plan.device_buffer is None:
        plan.upload(q.device, stream)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=q.device)
    need = plan.info().workspace_bytes
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(int(need), 256), dtype=torch.uint8, device=q.device)
    check(lib.dd_cascade_decode(C.byref(cfg), plan._h, _ptr(q), _ptr(kv_pages), _ptr(kv_scales),
                                _ptr(out), _ptr(lse), _ptr(workspace), workspace.numel(),
                                _stream(stream)), "dd_cascade_decode")
    return out, lse


def decode_paged(cfg: AttnConfig, q, kv_pages, page_indptr, page_indices, num_tokens,
                 max_pages: int, kv_scales=None, out=None, lse=None, workspace=None, stream=None):
    """FlashInfer-style batch decode with device-resident CSR page tables."""
    B = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(B, q.shape[1], dtype=torch.float32, device=q.device)
    need = lib.dd_decode_paged_workspace_size(C.byref(cfg), B, max_pages)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(int(need), 256), dtype=torch.uint8, device=q.device)
    check(lib.dd_decode_paged(C.byref(cfg), B, max_pages, _ptr(q), _ptr(kv_pages), _ptr(kv_scales),
                              _ptr(page_indptr), _ptr(page_indices), _ptr(num_tokens), _ptr(out),
                              _ptr(lse), _ptr(workspace), workspace.numel(), _stream(stream)),
          "dd_decode_paged")
    return out, lse


def workspace_status(workspace: torch.Tensor, stream=None) -> tuple[int, int]:
    code, aux = C.c_uint32(), C.c_uint32()
    check(lib.dd_workspace_status(_ptr(workspace), _stream(stream), C.byref(code), C.byref(aux)),
          "dd_workspace_status")
    return code.value, aux.value


def selftest_wait(workspace: torch.Tensor, limit_ns: int, stream=None) -> None:
    """Run the kernels' bounded wait out on purpose (dd_selftest_wait): the
    workspace then reports a wait timeout (status code 2)."""
    check(lib.dd_selftest_wait(_ptr(workspace), int(limit_ns), _stream(stream)), "dd_selftest_wait")


def merge_states(o_a, lse_a, o_b, lse_b, stream=None):
    """Batched merge_attention_outputs (cascade.rs:116-124) on the GPU."""
    n, D = o_a.shape[0], o_a.shape[-1]
    o = torch.empty_like(o_a)
    l = torch.empty_like(lse_a)
    check(lib.dd_merge_states(n, D, _ptr(o_a), _ptr(lse_a), _ptr(o_b), _ptr(lse_b), _ptr(o),
                              _ptr(l), _stream(stream)), "dd_merge_states")
    return o, l


# ------------------------------------------------------------- quantisation
def quant_config(fmt: str, num_kv_heads: int, head_dim: int, src_dtype=torch.bfloat16,
                 scale_mode: int = 0) -> QuantConfig:
    return QuantConfig(_KV_DTYPES[fmt], DTYPE_F32 if src_dtype == torch.float32 else DTYPE_BF16,
                       num_kv_heads, head_dim, PAGE_SIZE, scale_mode)


def quantize_kv_pages(pages: torch.Tensor, fmt: str, scale_mode: int = 0, stream=None,
                      codes: torch.Tensor | None = None, scales: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None):
    """Quantise a page pool [P][2][Hkv][16][D] (bf16 or f32) to E4M3 codes +
    per-head f32 scales ("e4m3") or E4M3 codes + E8M0 bytes ("mxfp8").
    codes / scales / workspace may be passed preallocated."""
    P, _, Hkv, _, D = pages.shape
    qc = quant_config(fmt, Hkv, D, pages.dtype, scale_mode)
    if codes is None:
        codes = torch.empty(pages.shape, dtype=torch.uint8, device=pages.device)
    if scales is None:
        if fmt == "e4m3":
            scales = torch.empty(2, Hkv, dtype=torch.float32, device=pages.device)
        else:
            scales = torch.empty(P, 2, Hkv, PAGE_SIZE, D // 32, dtype=torch.uint8, device=pages.device)
    need = max(int(lib.dd_quantize_workspace_size(C.byref(qc))), 256)
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(need, dtype=torch.uint8, device=pages.device)
    check(lib.dd_quantize_kv_pages(C.byref(qc), _ptr(pages), P, _ptr(codes), _ptr(scales), _ptr(ws),
                                   ws.numel(), _stream(stream)), "dd_quantize_kv_pages")
    return codes, scales


def dequantize_kv_pages(codes: torch.Tensor, scales: torch.Tensor, fmt: str,
                        out_dtype=torch.bfloat16, stream=None) -> torch.Tensor:
    P, _, Hkv, _, D = codes.shape
    qc = quant_config(fmt, Hkv, D)
    out = torch.empty(codes.shape, dtype=out_dtype, device=codes.device)
    check(lib.dd_dequantize_kv_pages(C.byref(qc), _ptr(codes), _ptr(scales), P, _ptr(out),
                                     DTYPE_F32 if out_dtype == torch.float32 else DTYPE_BF16,
                                     _stream(stream)), "dd_dequantize_kv_pages")
    return out


def append_kv_batch(cfg: AttnConfig, kv_pages: torch.Tensor, kv_scales: torch.Tensor | None,
                    page_ids: torch.Tensor, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    status: torch.Tensor | None = None, stream=None) -> None:
    """Append token i of k, v [n, Hkv, D] (bf16 or f32) to slot slots[i] of
    page page_ids[i] (device int tensors), quantizing for FP8 pools."""
    src = DTYPE_F32 if k.dtype == torch.float32 else DTYPE_BF16
    check(lib.dd_append_kv_batch(C.byref(cfg), _ptr(kv_pages), _ptr(kv_scales), k.shape[0],
                                 _ptr(page_ids), _ptr(slots), _ptr(k), _ptr(v), src, _ptr(status),
                                 _stream(stream)), "dd_append_kv_batch")


def copy_pages(cfg: AttnConfig, kv_pages: torch.Tensor, kv_scales: torch.Tensor | None,
               src: torch.Tensor, dst: torch.Tensor, status: torch.Tensor | None = None,
               stream=None) -> None:
    """Copy-on-write data copy: page dst[i] <- page src[i]."""
    check(lib.dd_copy_pages(C.byref(cfg), _ptr(kv_pages), _ptr(kv_scales), src.numel(), _ptr(src),
                            _ptr(dst), _ptr(status), _stream(stream)), "dd_copy_pages")


def scatter_head_shards(cfg: AttnConfig, world: int, gathered: torch.Tensor, out: torch.Tensor,
                        stream=None) -> torch.Tensor:
    check(lib.dd_scatter_head_shards(C.byref(cfg), world, out.shape[0], _ptr(gathered), _ptr(out),
                                     _stream(stream)), "dd_scatter_head_shards")
    return out


# ------------------------------------------------------------------ backend
class B200Backend:
    """AttentionBackend over a device KV page pool (see module docstring)."""

    def __init__(self, num_pages: int, num_kv_heads: int, head_dim: int, kv_dtype: str = "bf16",
                 device: str | torch.device = "cuda", gqa_map: int = GQA_TILED):
        if head_dim not in SUPPORTED_HEAD_DIMS:
            raise _lib.InvalidArgument(f"unsupported head_dim: {head_dim}, supported: [64, 128, 256]")
        if kv_dtype not in ("f32", "bf16"):
            raise _lib.InvalidArgument("the pool stores f32 or bf16 pages; quantize with quantize()")
        self.device = torch.device(device)
        self.num_pages = num_pages
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.gqa_map = gqa_map
        tdt = torch.float32 if kv_dtype == "f32" else torch.bfloat16
        self.pages = torch.zeros(num_pages, 2, num_kv_heads, PAGE_SIZE, head_dim, dtype=tdt,
                                 device=self.device)
        self.kv_dtype = kv_dtype
        self.codes = None
        self.scales = None
        self._ws: dict = {}

    # -- storage ----------------------------------------------------------
    def _cfg(self, config: AttentionConfig, q_dtype: torch.dtype) -> AttnConfig:
        if config.num_kv_heads != self.num_kv_heads or config.head_dim != self.head_dim:
            raise _lib.InvalidArgument("config does not match the KV pool")
        kvd = _KV_DTYPES[self.kv_dtype]
        qd = DTYPE_F32 if q_dtype == torch.float32 else DTYPE_BF16
        return make_config(config.num_heads, config.num_kv_heads, config.head_dim, self.num_pages,
                           kvd, qd, self.gqa_map, config.scale)

    def append_kv(self, key: torch.Tensor, value: torch.Tensor, block_table: BlockTable,
                  position: int) -> None:
        """backend.rs:285-301: store [1, Hkv, t, D] K/V in block_table[position // 16]."""
        block = block_table.get(position // PAGE_SIZE)
        if block is None:  # the reference silently ignores a missing block
            return
        k = key.reshape(self.num_kv_heads, -1, self.head_dim).to(self.pages.dtype).contiguous()
        v = value.reshape(self.num_kv_heads, -1, self.head_dim).to(self.pages.dtype).contiguous()
        cfg = make_config(self.num_kv_heads, self.num_kv_heads, self.head_dim, self.num_pages,
                          DTYPE_F32 if self.pages.dtype == torch.float32 else DTYPE_BF16)
        check(lib.dd_append_kv(C.byref(cfg), _ptr(self.pages), int(block), int(position),
                               int(k.shape[1]), _ptr(k), _ptr(v), _stream()), "dd_append_kv")
        self.codes = None  # quantised copy is stale

    def quantize(self, fmt: str, scale_mode: int = 0) -> None:
        """Switch decode to FP8 pages quantised from the current pool."""
        if self.pages.dtype != torch.bfloat16:
            raise _lib.InvalidArgument("quantize a bf16 pool")
        self.codes, self.scales = quantize_kv_pages(self.pages, fmt, scale_mode)
        self.kv_dtype = fmt

    # -- attention --------------------------------------------------------
    def prefill(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                block_table: BlockTable, config: AttentionConfig) -> torch.Tensor:
        """backend.rs:163-204: causal attention of query [1, Hq, S, D] over
        key / value [1, Hkv, S, D], over pages. block_table already counts the
        S new tokens: they are its last S, after prefix_len = num_tokens - S
        earlier tokens that every new token also sees (0 for the reference's
        dense prefill). Their K/V are stored into its pages (as append_kv
        would), then one causal plan runs over the pages."""
        S = query.shape[2]
        prefix = block_table.num_tokens() - S
        if prefix < 0:
            raise _lib.InvalidArgument("block_table must count the prefill tokens (num_tokens >= seq_len)")
        if block_table.num_blocks() * PAGE_SIZE < prefix + S:
            raise _lib.InvalidArgument("block_table has too few blocks for the prefill tokens")
        if S == 0:
            return query.clone()
        pos = torch.arange(prefix, prefix + S)
        blocks = torch.tensor(block_table.blocks(), dtype=torch.int32)
        page_ids = blocks[pos // PAGE_SIZE].to(self.device)
        slots = (pos % PAGE_SIZE).to(torch.int32).to(self.device)
        k = key.reshape(self.num_kv_heads, S, self.head_dim).transpose(0, 1).contiguous()
        v = value.reshape(self.num_kv_heads, S, self.head_dim).transpose(0, 1).contiguous()
        src_dt = torch.float32 if k.dtype == torch.float32 else torch.bfloat16
        k, v = k.to(src_dt), v.to(src_dt)
        pool_cfg = make_config(self.num_kv_heads, self.num_kv_heads, self.head_dim, self.num_pages,
                               DTYPE_F32 if self.pages.dtype == torch.float32 else DTYPE_BF16)
        append_kv_batch(pool_cfg, self.pages, None, page_ids, slots, k.to(self.pages.dtype),
                        v.to(self.pages.dtype))
        if self.codes is not None:  # FP8 pages: quantize the new tokens in place too
            fp8_cfg = make_config(self.num_kv_heads, self.num_kv_heads, self.head_dim, self.num_pages,
                                  _KV_DTYPES[self.kv_dtype])
            append_kv_batch(fp8_cfg, self.codes, self.scales, page_ids, slots, k, v)
        q = query.reshape(config.num_heads, S, config.head_dim).transpose(0, 1)
        qd = torch.float32 if q.dtype == torch.float32 else torch.bfloat16
        q = q.to(qd).contiguous()
        cfg = self._cfg(config, qd)
        plan = CascadePlan.prefill(cfg, [0, block_table.num_blocks()], block_table.blocks(), [prefix], [S])
        plan.upload(self.device)
        kv, sc = self._kv()
        ws = _alloc_ws(plan.info().workspace_bytes, self.device, self._ws)
        out, _ = cascade_decode(cfg, plan, q, kv, sc, workspace=ws)
        return out.transpose(0, 1).reshape(query.shape).to(query.dtype)

    def _kv(self):
        if self.kv_dtype in ("e4m3", "mxfp8"):
            return self.codes, self.scales
        return self.pages, None

    def decode_batch(self, queries: list, block_tables: list, config: AttentionConfig) -> list:
        """backend.rs:267-283, as one cascade launch over the batch."""
        if not queries:
            return []
        q = torch.stack([x.reshape(config.num_heads, config.head_dim) for x in queries])
        qd = torch.float32 if q.dtype == torch.float32 else torch.bfloat16
        q = q.to(qd).contiguous()
        cfg = self._cfg(config, qd)
        plan = CascadePlan.from_tables(cfg, block_tables)
        plan.upload(self.device)
        kv, sc = self._kv()
        ws = _alloc_ws(plan.info().workspace_bytes, self.device, self._ws)
        out, _ = cascade_decode(cfg, plan, q, kv, sc, workspace=ws)
        return [out[i].reshape(queries[i].shape).to(queries[i].dtype) for i in range(len(queries))]

    def decode(self, query: torch.Tensor, block_table: BlockTable,
               config: AttentionConfig) -> torch.Tensor:
        """backend.rs:206-265."""
        return self.decode_batch([query], [block_table], config)[0]
