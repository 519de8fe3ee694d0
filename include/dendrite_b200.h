/*
 * dendrite_b200 — C ABI of the B200 (sm_100a) paged cascade decode-attention
 * path and its FP8 / MXFP8 KV-page codec.
 *
 * This is the kernel layer that sits in the slot of Dendrite's `dendrite-ffi`
 * crate (crates/dendrite-ffi/src/flashinfer/*.rs). Every entry point is a
 * plain C function over raw pointers and sizes; no C++ or torch types cross
 * the boundary, so it binds from Rust (`extern "C"`), Python (ctypes) or C.
 *
 * Conventions (shared by all entry points)
 *  - Return value: dd_status. 0 = ok. The non-zero codes map one-to-one onto
 *    the reference's `FfiError` variants (crates/dendrite-ffi/src/error.rs:9-30):
 *      DD_ERR_INVALID_ARGUMENT -> FfiError::InvalidArgument
 *      DD_ERR_CUDA             -> FfiError::CudaError
 *      DD_ERR_NOT_AVAILABLE    -> FfiError::NotAvailable
 *      DD_ERR_ALLOCATION       -> FfiError::AllocationFailed
 *      DD_ERR_WORKSPACE        -> FfiError::InvalidArgument (workspace too small)
 *    `dd_last_error()` returns a human-readable message for the calling thread.
 *  - Ownership: the caller owns every device buffer. The hot calls never
 *    allocate device memory; scratch space is the caller's `workspace`, sized
 *    by the matching `*_workspace_size` query (as `workspace_size()` is in
 *    crates/dendrite-ffi/src/flashinfer/batch_decode.rs:57-59).
 *  - Asynchrony: kernels are enqueued on the given stream (NULL = legacy
 *    default stream). Launch errors are returned; faults surface at the next
 *    synchronisation, as with any CUDA library.
 *  - Threading: functions are stateless and re-entrant. A dd_plan may be used
 *    from one thread at a time.
 *
 * Memory layouts
 *  - KV page pool: [num_pages][2 (K,V)][num_kv_heads][16][head_dim], the
 *    layout of a Dendrite `Page` (crates/dendrite-core/src/cache/paged.rs:57,
 *    90-94). Element type per dd_attn_config.kv_dtype:
 *      DD_DTYPE_F32, DD_DTYPE_BF16: values;
 *      DD_DTYPE_E4M3:  one FP8 E4M3 code per element, with kv_scales =
 *                      float[2][num_kv_heads] (one scale per K/V x KV head);
 *      DD_DTYPE_MXFP8: one FP8 E4M3 code per element, with kv_scales =
 *                      uint8 E8M0 [num_pages][2][num_kv_heads][16][head_dim/32]
 *                      (one shared exponent per 32 consecutive elements of a
 *                      token's head vector, OCP MX v1.0).
 *    Slots of a sequence's last page beyond its valid tokens must hold finite
 *    values (their scores are masked, but the kernels multiply their zero
 *    weights by the stored V); Dendrite's pages start zeroed
 *    (Tensor::zeros, cache/paged.rs:86-92) and the quantize / append entry
 *    points here write only finite codes.
 *  - Queries / outputs: [batch][num_qo_heads][head_dim] (q_dtype, out in
 *    q_dtype). lse: float [batch][num_qo_heads], natural-log log-sum-exp of
 *    the scaled scores, the convention of merge_attention_outputs
 *    (crates/dendrite-ffi/src/flashinfer/cascade.rs:116-124).
 *  - Block tables: CSR. Query b uses block ids
 *    block_ids[block_indptr[b] .. block_indptr[b+1]) and its first
 *    num_tokens[b] tokens (16 per block; the last block may be partial).
 *  - GQA: query head h reads KV head (h % num_kv_heads) under
 *    DD_GQA_TILED — what ReferenceBackend's `Tensor::repeat` tiling does
 *    (crates/dendrite-core/src/attention/backend.rs:245-252) — or
 *    (h / (num_qo_heads/num_kv_heads)) under DD_GQA_GROUPED (the Llama
 *    model layer's expand/reshape, crates/dendrite-core/src/model/layer.rs:321-340).
 */
#ifndef DENDRITE_B200_H
#define DENDRITE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* dd_stream_t; /* == cudaStream_t */

typedef enum dd_status {
  DD_OK = 0,
  DD_ERR_INVALID_ARGUMENT = 1,
  DD_ERR_CUDA = 2,
  DD_ERR_NOT_AVAILABLE = 3,
  DD_ERR_ALLOCATION = 4,
  DD_ERR_WORKSPACE = 5
} dd_status;

/* Element types. 0 and 1 keep the reference's dtype codes
 * (crates/dendrite-ffi/src/flashinfer/batch_decode.rs:19-20: 0=f16, 1=bf16). */
typedef enum dd_dtype {
  DD_DTYPE_F16 = 0,   /* accepted by the config but not implemented: NOT_AVAILABLE */
  DD_DTYPE_BF16 = 1,
  DD_DTYPE_F32 = 2,
  DD_DTYPE_E4M3 = 3,  /* KV only: FP8 E4M3 codes + per-(K/V, head) f32 scale */
  DD_DTYPE_MXFP8 = 4  /* KV only: FP8 E4M3 codes + E8M0 scale per 32 elements */
} dd_dtype;

typedef enum dd_gqa_map { DD_GQA_TILED = 0, DD_GQA_GROUPED = 1 } dd_gqa_map;

/* Replaces AttentionConfig (crates/dendrite-core/src/attention/backend.rs:17-58)
 * together with BatchDecodeConfig / CascadeConfig
 * (crates/dendrite-ffi/src/flashinfer/batch_decode.rs:7-21, cascade.rs:7-20).
 * scale <= 0 selects 1/sqrt(head_dim) computed in f32 (backend.rs:37). */
typedef struct dd_attn_config {
  int32_t num_qo_heads;
  int32_t num_kv_heads;
  int32_t head_dim;   /* 64, 128 or 256 (flashinfer/mod.rs:20) */
  int32_t page_size;  /* must be 16 (flashinfer/mod.rs:14, cache/mod.rs:61) */
  int32_t kv_dtype;   /* dd_dtype */
  int32_t q_dtype;    /* DD_DTYPE_BF16 or DD_DTYPE_F32 */
  int32_t gqa_map;    /* dd_gqa_map */
  int32_t num_pages;  /* pool size; block ids must be < num_pages */
  float scale;
} dd_attn_config;

/* Library version / last error --------------------------------------------- */
const char* dd_version(void);
const char* dd_last_error(void);
/* Validates cfg against the rules of BatchDecodeKernel::new
 * (crates/dendrite-ffi/src/flashinfer/batch_decode.rs:31-55). */
int dd_validate_config(const dd_attn_config* cfg);

/* Cascade plan -------------------------------------------------------------
 * The batch builder's prefix/suffix plan. Built on the host from the decode
 * batch's block tables: the trie over block-id sequences is exactly the
 * copy-on-write sharing of TreeState::fork (crates/dendrite-core/src/tree/state.rs:49-84,
 * BlockTable::fork crates/dendrite-core/src/cache/block_table.rs:97-103), so
 * every node of the plan is a run of pages shared by a contiguous range of
 * queries. Replaces the per-query gather loop of ReferenceBackend::decode_batch
 * (backend.rs:267-283) and the shared/unique split that CascadeAttention::run
 * documents (crates/dendrite-ffi/src/flashinfer/cascade.rs:69-83). */
typedef struct dd_plan dd_plan;

typedef struct dd_plan_options {
  int32_t share_prefixes;  /* 1: cascade over shared prefixes; 0: flat per-query plan */
  int32_t max_chunk_pages; /* 0 = automatic split-K chunking */
  int32_t use_tensor_cores;/* 1 (default): tcgen05 path for nodes with many rows */
  int32_t cta_pairs;        /* 1: nodes of > 256 rows run on CTA pairs (cta_group::2
                             * tcgen05 kernel, bf16 only); 0 (default): one-SM kernel */
  int32_t tc_sms;           /* CTAs of the tcgen05 kernel, each running a scheduled list
                             * of work items: 0 (default) = one per SM; N > 0 = N (the
                             * streaming kernel starts on the other SMs); -1 = one CTA
                             * per work item with the older split-K rule */
} dd_plan_options;

typedef struct dd_plan_info {
  int32_t batch_size;
  int32_t num_nodes;       /* cascade nodes (shared runs of pages) */
  int32_t num_items;       /* kernel work items */
  int32_t max_depth;       /* longest root-to-leaf node path */
  int64_t kv_tokens;       /* unique KV tokens read (each shared node once) */
  int64_t kv_tokens_flat;  /* tokens a non-sharing decode would read */
  size_t workspace_bytes;  /* required size of `workspace` */
  size_t device_bytes;     /* required size of the buffer given to dd_plan_upload */
  /* Unique KV tokens read by each attention kernel: [0] CUDA-core kernel,
   * [1] streaming tensor-core (mma) kernel, [2] tcgen05 kernel (wide nodes),
   * [3] tcgen05 kernel on CTA pairs (the widest nodes), [4] unused (0). */
  int64_t kv_tokens_by_kernel[5];
  /* Sum over tcgen05 nodes and KV heads of (query rows x tokens): the
   * kernel's 4 * head_dim FLOPs per unit (Q.K^T and P.V). */
  int64_t tc_row_tokens;
  int32_t tc_ctas;         /* CTAs of the tcgen05 launch (0: no tcgen05 work) */
} dd_plan_info;

int dd_plan_create(const dd_attn_config* cfg, int32_t batch_size,
                   const int32_t* block_indptr, const uint32_t* block_ids,
                   const int32_t* num_tokens, const dd_plan_options* opts,
                   dd_plan** out_plan);
void dd_plan_destroy(dd_plan* plan);
/* Causal prefill plan over paged KV (chunked prefill of branch suffixes):
 * sequence s holds prefix_len[s] + num_new[s] tokens in its block table
 * block_ids[block_indptr[s] .. block_indptr[s+1]), the last num_new[s] of
 * them new (their K/V already stored, e.g. by dd_append_kv_batch). Its new
 * token i is a query that sees tokens [0, prefix_len[s] + i] of the sequence;
 * queries are numbered sequence-major, so q / out of dd_cascade_decode are
 * [sum(num_new)][num_qo_heads][head_dim]. With prefix_len = 0 this is
 * ReferenceBackend::prefill's causal attention
 * (crates/dendrite-core/src/attention/backend.rs:163-204) over pages; the
 * stub it replaces is BatchPrefillKernel::run
 * (crates/dendrite-ffi/src/flashinfer/batch_prefill.rs). Each sequence's
 * pages are read once per row tile of its queries; dd_plan_rebuild turns the
 * plan back into a decode plan. */
int dd_plan_create_prefill(const dd_attn_config* cfg, int32_t num_seqs,
                           const int32_t* block_indptr, const uint32_t* block_ids,
                           const int32_t* prefix_len, const int32_t* num_new,
                           const dd_plan_options* opts, dd_plan** out_plan);
/* Re-plans an existing plan for a new decode batch (same config and
 * options), reusing its host memory: the per-step call of an engine whose
 * tree grows by one token per leaf per step. The device image must be
 * uploaded again (dd_plan_upload) before the next dd_cascade_decode. On
 * error the plan is left empty (batch 0). No reference counterpart. */
int dd_plan_rebuild(dd_plan* plan, int32_t batch_size, const int32_t* block_indptr,
                    const uint32_t* block_ids, const int32_t* num_tokens);
/* Advances a decode plan by one decode step in place, the per-step call of
 * an engine whose leaves each grow by a token (the scheduler's plan cache):
 * query b (batch order) gained tokens_added[b] tokens (0 or 1); a token that
 * starts a new block went to block new_block[b] (read only for those). In
 * place only for queries that own their last pages (a leaf of the plan's
 * tree with no other query): their nodes gain the token / block and their
 * items are re-cut; the device image must be uploaded again (its size,
 * dd_plan_get_info().device_bytes, can grow by the moved page runs): a
 * successful advance forgets the previous upload, so dd_cascade_decode
 * returns DD_ERR_INVALID_ARGUMENT until the plan is uploaded again. Returns
 * DD_ERR_NOT_AVAILABLE, with the plan unchanged, when some query shares its
 * last pages (a fresh fork, a copy-on-write pending), for prefill and flat
 * plans, or when the page list needs compacting: the caller then re-plans
 * with dd_plan_rebuild from the full block tables. No reference counterpart
 * (the reference re-reads every block table per query and step). */
int dd_plan_advance(dd_plan* plan, const int32_t* tokens_added, const uint32_t* new_block);
int dd_plan_get_info(const dd_plan* plan, dd_plan_info* info);
/* Copies the plan's arrays into caller-owned device memory (>= device_bytes,
 * 256-byte aligned). Must be called before dd_cascade_decode. The copy is
 * asynchronous on `stream`, from a pinned host buffer the plan keeps (grown
 * with cudaHostAlloc when the plan grows; freed by dd_plan_destroy); the next
 * upload of the same plan first waits for this copy to finish. */
int dd_plan_upload(dd_plan* plan, void* device_buf, size_t bytes, dd_stream_t stream);
/* Host view of the plan's nodes, for tests and tooling. Each array may be
 * NULL; non-NULL arrays have num_nodes entries, except node_pages: every
 * node's pages one node after another (sum of node_page_count entries; pass
 * NULL and read node_page_count to size it), node_page_offset indexing it. */
int dd_plan_export_nodes(const dd_plan* plan, int32_t* node_parent,
                         int32_t* node_q_begin, int32_t* node_num_q,
                         int32_t* node_num_tokens, int32_t* node_page_offset,
                         int32_t* node_page_count, uint32_t* node_pages,
                         int32_t* query_order);

/* Cascade decode over a plan. Replaces CascadeAttention::run
 * (crates/dendrite-ffi/src/flashinfer/cascade.rs:84-101) and, via a plan
 * made with share_prefixes = 0, BatchDecodeKernel::run (batch_decode.rs:86-101).
 * q: [batch][Hq][D]; out: [batch][Hq][D] (q_dtype); lse may be NULL.
 * kv_scales: see "Memory layouts" (NULL for F32/BF16). */
int dd_cascade_decode(const dd_attn_config* cfg, const dd_plan* plan,
                      const void* q, const void* kv_pages, const void* kv_scales,
                      void* out, float* lse, void* workspace, size_t workspace_bytes,
                      dd_stream_t stream);

/* Paged batch decode with device-resident CSR page tables and no plan (no
 * prefix sharing): the FlashInfer-style entry point of
 * BatchDecodeKernel::run (crates/dendrite-ffi/src/flashinfer/batch_decode.rs:86-101).
 * page_indptr/page_indices/num_tokens are device arrays (int32). Instead of
 * last_page_len (0 for a full page in PageTable::last_page_len, paged.rs:384-390)
 * it takes num_tokens per sequence. max_pages_per_seq bounds the split-K grid. */
size_t dd_decode_paged_workspace_size(const dd_attn_config* cfg, int32_t batch_size,
                                      int32_t max_pages_per_seq);
int dd_decode_paged(const dd_attn_config* cfg, int32_t batch_size, int32_t max_pages_per_seq,
                    const void* q, const void* kv_pages, const void* kv_scales,
                    const int32_t* page_indptr, const int32_t* page_indices,
                    const int32_t* num_tokens, void* out, float* lse,
                    void* workspace, size_t workspace_bytes, dd_stream_t stream);

/* Reads the device status words at the head of a workspace used by the last
 * decode on `stream` (synchronises the stream). code 0 = no error;
 * 1 = a block id >= num_pages was met in a device-side page table (the page
 * was skipped, as ReferenceBackend::decode skips blocks without KV,
 * backend.rs:228-234; aux = the id); 2 = a kernel's bounded wait timed out. */
int dd_workspace_status(const void* workspace, dd_stream_t stream, uint32_t* code, uint32_t* aux);

/* Failure-path self-test: runs the kernels' bounded mbarrier wait on a
 * barrier nothing arrives on, with limit_ns (<= 2 s) instead of 2 s. The
 * kernel gives up, records status code 2 (a bounded wait timed out) in the
 * workspace header (>= 256 bytes; read with dd_workspace_status) and
 * returns: the context stays
 * usable. For tests of the failure detection. */
int dd_selftest_wait(void* workspace, uint64_t limit_ns, dd_stream_t stream);

/* 1 when the tcgen05 (TMEM) kernel for wide shared nodes is compiled in. */
int dd_tc_available(void);

/* Instrumentation (no reference counterpart; the reference has no tracing,
 * its `tracing` dependency is unused). dd_launch_count: kernels launched by
 * this library since load. dd_profile_enable(1): record a CUDA event pair on
 * the launching stream around every launch; dd_profile_read: synchronise on
 * them and return, per kernel family k < n (0 CUDA-core attention, 1 mma
 * attention, 2 tcgen05 attention, 3 merge, 4 quantize/dequantize, 5 other),
 * the summed milliseconds and launch counts since the previous read. */
uint64_t dd_launch_count(void);
void dd_profile_enable(int on);
int dd_profile_read(double* ms, int64_t* launches, int32_t n);

/* Paged batch decode that allocates nothing. No counterpart in the reference.
 * For callers that cannot allocate device memory for scratch — a plugin that
 * receives only input/output pointers from a host engine owning all device
 * memory, or a decode loop that must not call cudaMalloc — this variant of
 * dd_decode_paged takes no workspace: its scratch (split-K partial states and
 * status words) lives in one static 4 MiB device array inside this library,
 * held on every GPU that loads the library until the process exits. Arguments
 * and results are dd_decode_paged's. A batch whose scratch
 * (dd_decode_paged_workspace_size) exceeds 4 MiB is rejected with
 * DD_ERR_WORKSPACE. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. Every call shares the one array, so calls
 * whose executions overlap on the GPU (different streams, or different host
 * threads on one device) race and corrupt each other's results: serialise
 * them. The device address is looked up once per device and kept for the
 * life of the process: do not use this entry point on a device after
 * cudaDeviceReset (or any other destruction of its primary context) in the
 * same process. The function calls no cudaMalloc / cudaFree. */
int dd_decode_paged_static(const dd_attn_config* cfg, int32_t batch_size,
                           int32_t max_pages_per_seq, const void* q, const void* kv_pages,
                           const void* kv_scales, const int32_t* page_indptr,
                           const int32_t* page_indices, const int32_t* num_tokens, void* out,
                           float* lse, dd_stream_t stream);
/* Device status of the last dd_decode_paged_static call on the current
 * device, as dd_workspace_status reports it for a caller workspace (0 = OK;
 * otherwise an error code such as a bounded-wait timeout or an out-of-range
 * page id, with its detail in *aux). Reads the status words at the head of
 * the static scratch on `stream` and synchronises it. No counterpart in the
 * reference. */
int dd_decode_paged_static_status(dd_stream_t stream, uint32_t* code, uint32_t* aux);

/* Merge of attention states: (o_a, lse_a) (+) (o_b, lse_b) -> (o, lse), f32,
 * natural-log LSE, element-wise over n rows of head_dim. The batched form of
 * merge_attention_outputs (crates/dendrite-ffi/src/flashinfer/cascade.rs:116-124).
 * o may alias o_a or o_b; lse may not alias lse_a or lse_b. */
int dd_merge_states(int32_t n, int32_t head_dim, const float* o_a, const float* lse_a,
                    const float* o_b, const float* lse_b, float* o, float* lse,
                    dd_stream_t stream);

/* KV-page append (page scatter). Replaces ReferenceBackend::append_kv
 * (crates/dendrite-core/src/attention/backend.rs:285-301) for the paged pool:
 * writes t tokens of k, v ([num_kv_heads][t][head_dim], kv_dtype F32 or BF16)
 * into page `block_id` at token slots position%16 .. position%16 + t - 1
 * (requires position%16 + t <= 16). */
int dd_append_kv(const dd_attn_config* cfg, void* kv_pages, uint32_t block_id,
                 int32_t position, int32_t t, const void* k, const void* v,
                 dd_stream_t stream);

/* Decode-step append of n tokens in one launch (no reference counterpart in
 * batched form; per token it is ReferenceBackend::append_kv, backend.rs:285-301):
 * token i of k, v ([n][num_kv_heads][head_dim], src_dtype F32 or BF16) goes
 * to token slot slots[i] (0..15) of page page_ids[i] (device arrays), in the
 * pool's storage type: values for F32/BF16 pages (bf16 RNE), RNE-saturating
 * E4M3 of x / kv_scales[kv][h] for per-head E4M3 pages (the pool's scales
 * are used as they are), E4M3 codes + E8M0 exponent per 32-element block for
 * MXFP8 pages (as dd_quantize_kv_pages writes them). Out-of-range page ids or
 * slots are skipped; if `status` (device, 2 x uint32, may be NULL) is given,
 * status[0] = 1 and status[1] = the first such token. */
int dd_append_kv_batch(const dd_attn_config* cfg, void* kv_pages, void* kv_scales, int32_t n,
                       const uint32_t* page_ids, const int32_t* slots, const void* k,
                       const void* v, int32_t src_dtype, uint32_t* status, dd_stream_t stream);

/* Copy-on-write data copy: page dst[i] <- page src[i] for i < n (device
 * arrays; all K/V data of the page and, for MXFP8, its exponent bytes). The
 * reference's BlockPool::copy_on_write (crates/dendrite-core/src/cache/pool.rs:88-91)
 * only swaps ids. Invalid ids are skipped (status[0] = 2, status[1] = i). */
int dd_copy_pages(const dd_attn_config* cfg, void* kv_pages, void* kv_scales, int32_t n,
                  const uint32_t* src, const uint32_t* dst, uint32_t* status, dd_stream_t stream);

/* KV-page quantization ------------------------------------------------------
 * Replaces QuantizedTensor::quantize / dequantize
 * (crates/dendrite-core/src/quantization/fp8.rs:103-152) with real E4M3 codes.
 *  DD_DTYPE_E4M3: scale[kv][h] = amax over every token of the pool for that
 *    K/V and KV head, times f32(1/448) (scale_mode 0: candle's `tensor / f64`
 *    lowers to an affine multiply by the reciprocal) or divided by 448
 *    (scale_mode 1); amax == 0 gives scale 1. code = RNE-saturating E4M3 of
 *    x / scale (fp8.rs:125-130 with the clamp at +-448 made a rounding).
 *  DD_DTYPE_MXFP8: per 32 elements, shared exponent
 *    e = max(-127, floor(log2(amax)) - 8), E8M0 byte e + 127;
 *    code = RNE-saturating E4M3 of x * 2^-e (OCP MX v1.0, block size 32 as in
 *    QuantConfig, crates/dendrite-core/src/quantization/mod.rs:97,133-140).
 * src: [num_pages][2][Hkv][16][D] bf16 (or f32 with src_dtype F32).
 * codes: uint8, same element layout. scales: float[2][Hkv] (E4M3) or
 * uint8 [num_pages][2][Hkv][16][D/32] (MXFP8).
 * The E4M3 path needs a workspace of dd_quantize_workspace_size bytes. */
typedef struct dd_quant_config {
  int32_t format;      /* DD_DTYPE_E4M3 or DD_DTYPE_MXFP8 */
  int32_t src_dtype;   /* DD_DTYPE_BF16 or DD_DTYPE_F32 */
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t page_size;   /* 16 */
  int32_t scale_mode;  /* E4M3 only: 0 = amax * f32(1/448), 1 = amax / 448 */
} dd_quant_config;

size_t dd_quantize_workspace_size(const dd_quant_config* qc);
int dd_quantize_kv_pages(const dd_quant_config* qc, const void* src, int64_t num_pages,
                         uint8_t* codes, void* scales, void* workspace, size_t ws_bytes,
                         dd_stream_t stream);
/* Round trip: codes (+scales) -> dst (DD_DTYPE_BF16 RNE or DD_DTYPE_F32). */
int dd_dequantize_kv_pages(const dd_quant_config* qc, const uint8_t* codes,
                           const void* scales, int64_t num_pages, void* dst,
                           int32_t dst_dtype, dd_stream_t stream);

/* KV-head split of one long tree with the join fused into the decode: as
 * dd_cascade_decode on this rank's shard (cfg_local = Hq/world query heads
 * over Hkv/world KV heads, plan built with cfg_local, q_local / kv_local /
 * scales_local the rank's heads as dd_scatter_head_shards documents), but the
 * final merge writes each output row at its global head of EVERY rank's
 * output [batch][num_qo_heads][head_dim]: peer_out is a DEVICE array of
 * `world` device pointers to those buffers (peer memory mapped into this
 * process, e.g. a symmetric-memory allocation; NVLink stores, no collective
 * library). lse_local [batch][Hq/world] stays local. The caller synchronises
 * the ranks after the call (before reading the output) and before a rank's
 * next call can overwrite a buffer another rank still reads. Replaces the
 * decode + NCCL all-gather + reorder of the head split; no reference
 * counterpart (the reference runs no multi-GPU attention). */
int dd_cascade_decode_shards(const dd_attn_config* cfg_local, const dd_plan* plan,
                             const void* q_local, const void* kv_local, const void* scales_local,
                             void* const* peer_out, int32_t world, int32_t rank,
                             int32_t num_qo_heads, int32_t num_kv_heads, float* lse_local,
                             void* workspace, size_t workspace_bytes, dd_stream_t stream);

/* Multi-GPU helper for the KV-head split of one long tree: after an
 * all-gather of per-rank outputs gathered[rank][batch][Hq/world][D], writes
 * out[batch][Hq][D]. rank r owns KV heads [r*Hkv/world, (r+1)*Hkv/world) and
 * the query heads that map to them under cfg->gqa_map. Both buffers must be
 * 16-byte aligned (rows move as 16-byte vectors). */
int dd_scatter_head_shards(const dd_attn_config* cfg, int32_t world, int32_t batch_size,
                           const void* gathered, void* out, dd_stream_t stream);

/* The collective of that split: ncclAllGather of this rank's local_out
 * [batch][Hq/world][D] (cfg->q_dtype, bf16 or f32) into gathered (device
 * scratch of world * batch * (Hq/world) * D elements) on `stream`, then
 * dd_scatter_head_shards into out [batch][Hq][D]. nccl_comm is the caller's
 * ncclComm_t over the `world` ranks (rank order = KV-head-group order); the
 * library does not link NCCL, it calls the NCCL already loaded in the
 * process (else libnccl.so.2), and returns DD_ERR_NOT_AVAILABLE without one.
 * No reference counterpart: the reference has no multi-GPU attention; this is
 * the all-gather its scope (one long tree split by KV-head group) calls for. */
int dd_allgather_heads(void* nccl_comm, const dd_attn_config* cfg, int32_t world,
                       int32_t batch_size, const void* local_out, void* gathered, void* out,
                       dd_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* DENDRITE_B200_H */
