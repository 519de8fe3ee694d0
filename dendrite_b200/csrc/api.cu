// C-ABI entry points: plan upload, cascade decode, flat paged decode, KV
// append, head-shard scatter. Kernel selection lives here; the kernels are in
// attn_simple.cu, attn_mma.cu, attn_tc.cu, attn_tc2.cu (CTA pairs, opt-in)
// and merge.cu; the planner is in
// planner.cpp, the quantizer in quant.cu, batched appends and page copies in
// append.cu, the head all-gather in collective.cu.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "dd_device.cuh"

namespace dd {
cudaError_t launch_attn_simple(const AttnArgs& a, dim3 grid, cudaStream_t st);
int launch_attn_mma(const AttnArgs& a, int64_t num_pages, cudaStream_t st, bool after_tc);
bool mma_supported(int D, int kv_dtype);
int launch_attn_tc(const AttnArgs& a, int64_t num_pages, int grid, cudaStream_t st);
int launch_attn_tc2(const AttnArgs& a, int64_t num_pages, int num_items, cudaStream_t st);
cudaError_t launch_merge(const MergeArgs& a, cudaStream_t st);

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(DD_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static AttnArgs base_args(const dd_attn_config* c, const void* q, const void* kv,
                          const void* scales, void* ws, size_t nslots) {
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = q;
  a.kv = kv;
  a.scales = scales;
  a.err = reinterpret_cast<WsHeader*>(ws);
  a.part_o = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kWsHeaderBytes);
  a.part_lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.part_o) +
                                        align_up(nslots * c->head_dim * sizeof(float), kAlign));
  a.Hq = c->num_qo_heads;
  a.Hkv = c->num_kv_heads;
  a.g = c->num_qo_heads / c->num_kv_heads;
  a.D = c->head_dim;
  a.kv_dtype = c->kv_dtype;
  a.q_dtype = c->q_dtype;
  a.gqa_map = c->gqa_map;
  a.num_pages = c->num_pages;
  const float scale = c->scale > 0.f ? c->scale : 1.0f / std::sqrt((float)c->head_dim);
  a.scale_log2 = scale * kLog2e;
  return a;
}

static int check_kv_ptrs(const dd_attn_config* c, const void* q, const void* kv,
                         const void* scales, const void* out) {
  if (!q || !out) return fail(DD_ERR_INVALID_ARGUMENT, "q / out is NULL");
  if (!kv && c->num_pages > 0) return fail(DD_ERR_INVALID_ARGUMENT, "kv_pages is NULL");
  if ((c->kv_dtype == DD_DTYPE_E4M3 || c->kv_dtype == DD_DTYPE_MXFP8) && !scales)
    return fail(DD_ERR_INVALID_ARGUMENT, "FP8 KV pages need kv_scales");
  if (((uintptr_t)kv & 15) || ((uintptr_t)q & 15))
    return fail(DD_ERR_INVALID_ARGUMENT, "kv_pages and q must be 16-byte aligned");
  return DD_OK;
}

static bool same_shape(const dd_attn_config& a, const dd_attn_config& b) {
  return a.num_qo_heads == b.num_qo_heads && a.num_kv_heads == b.num_kv_heads &&
         a.head_dim == b.head_dim && a.kv_dtype == b.kv_dtype && a.q_dtype == b.q_dtype &&
         a.gqa_map == b.gqa_map && a.num_pages == b.num_pages;
}

static int flat_nsplit(const dd_attn_config* c, int32_t B, int32_t max_pages) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int g = c->num_qo_heads / c->num_kv_heads;
  const int64_t base = (int64_t)std::max(B, 1) * c->num_kv_heads * ((g + 63) / 64);
  int64_t ns = (2 * (int64_t)sms + base - 1) / base;
  ns = std::min<int64_t>(ns, std::max<int64_t>(1, (max_pages + 3) / 4));
  return (int)std::max<int64_t>(1, std::min<int64_t>(ns, 64));
}

}  // namespace dd

using namespace dd;

namespace dd {
void release_staging(dd_plan* p) {
  if (p->staging_event) {
    cudaEventSynchronize((cudaEvent_t)p->staging_event);
    cudaEventDestroy((cudaEvent_t)p->staging_event);
  }
  if (p->staging) cudaFreeHost(p->staging);
  p->staging = nullptr;
  p->staging_event = nullptr;
  p->staging_bytes = 0;
  p->staging_device = -1;
}
}  // namespace dd

extern "C" int dd_plan_upload(dd_plan* p, void* buf, size_t bytes, dd_stream_t stream) {
  if (!p || !buf) return fail(DD_ERR_INVALID_ARGUMENT, "NULL argument");
  if (bytes < p->image.size()) return fail(DD_ERR_WORKSPACE, "plan device buffer too small");
  if ((uintptr_t)buf & (kAlign - 1)) return fail(DD_ERR_INVALID_ARGUMENT, "plan buffer must be 256-byte aligned");
  // The image goes through a pinned copy kept by the plan: a copy from
  // pageable memory would first wait for all work queued on the stream (the
  // caller's query upload, say) and stall the host. The previous upload's
  // copy must have left the staging buffer before it is overwritten.
  const size_t n = p->image.size();
  int dev = 0;
  cudaGetDevice(&dev);
  if (p->staging_event && p->staging_device != dev) release_staging(p);
  if (p->staging_event) cudaEventSynchronize((cudaEvent_t)p->staging_event);
  if (p->staging_bytes < n) {
    if (p->staging) cudaFreeHost(p->staging);
    p->staging = nullptr;
    p->staging_bytes = 0;
    const size_t want = n + n / 2;
    if (cudaHostAlloc(&p->staging, want, cudaHostAllocDefault) == cudaSuccess) {
      p->staging_bytes = want;
    } else {
      cudaGetLastError();
      p->staging = nullptr;
    }
  }
  if (p->staging && !p->staging_event) {
    cudaEvent_t ev;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess) {
      p->staging_event = ev;
      p->staging_device = dev;
    } else {
      cudaGetLastError();
    }
  }
  cudaError_t e;
  if (p->staging && p->staging_event) {
    std::memcpy(p->staging, p->image.data(), n);
    e = cudaMemcpyAsync(buf, p->staging, n, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaEventRecord((cudaEvent_t)p->staging_event, (cudaStream_t)stream);
  } else {
    // No pinned memory to be had: the plain (stream-ordered, host-blocking) copy.
    e = cudaMemcpyAsync(buf, p->image.data(), n, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "plan upload");
  p->device_base = buf;
  cudaGetDevice(&p->device_id);
  return DD_OK;
}

// Rank placement of a head-split decode whose merge writes into peer memory.
struct PeerOut {
  void* const* ptrs;
  int32_t world, rank, Hq_global, Hkv_global;
};

static int cascade_decode_impl(const dd_attn_config* cfg, const dd_plan* p, const void* q,
                               const void* kv, const void* scales, void* out, float* lse,
                               void* ws, size_t ws_bytes, dd_stream_t stream, const PeerOut* po);

extern "C" int dd_cascade_decode(const dd_attn_config* cfg, const dd_plan* p, const void* q,
                                 const void* kv, const void* scales, void* out, float* lse,
                                 void* ws, size_t ws_bytes, dd_stream_t stream) {
  return cascade_decode_impl(cfg, p, q, kv, scales, out, lse, ws, ws_bytes, stream, nullptr);
}

extern "C" int dd_cascade_decode_shards(const dd_attn_config* cfg_local, const dd_plan* p,
                                        const void* q_local, const void* kv_local,
                                        const void* scales_local, void* const* peer_out,
                                        int32_t world, int32_t rank, int32_t num_qo_heads,
                                        int32_t num_kv_heads, float* lse_local, void* ws,
                                        size_t ws_bytes, dd_stream_t stream) {
  int rc = check_config(cfg_local);
  if (rc) return rc;
  if (!peer_out) return fail(DD_ERR_INVALID_ARGUMENT, "peer_out is NULL");
  if (world < 1 || rank < 0 || rank >= world) return fail(DD_ERR_INVALID_ARGUMENT, "bad world / rank");
  if (num_kv_heads != cfg_local->num_kv_heads * world || num_qo_heads != cfg_local->num_qo_heads * world)
    return fail(DD_ERR_INVALID_ARGUMENT, "global head counts must be the local ones times world");
  const PeerOut po{peer_out, world, rank, num_qo_heads, num_kv_heads};
  // The local output buffer is not written; q_local stands in for the
  // pointer checks.
  return cascade_decode_impl(cfg_local, p, q_local, kv_local, scales_local,
                             const_cast<void*>(q_local), lse_local, ws, ws_bytes, stream, &po);
}

static int cascade_decode_impl(const dd_attn_config* cfg, const dd_plan* p, const void* q,
                               const void* kv, const void* scales, void* out, float* lse,
                               void* ws, size_t ws_bytes, dd_stream_t stream, const PeerOut* po) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (!p) return fail(DD_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (!same_shape(*cfg, p->cfg)) return fail(DD_ERR_INVALID_ARGUMENT, "config differs from the plan's");
  if (!p->device_base) return fail(DD_ERR_INVALID_ARGUMENT, "plan was not uploaded (dd_plan_upload)");
  if (p->batch_size == 0) return DD_OK;
  rc = check_kv_ptrs(cfg, q, kv, scales, out);
  if (rc) return rc;
  const size_t need = plan_workspace_bytes(p);
  if (!ws || ws_bytes < need) return fail(DD_ERR_WORKSPACE, "workspace smaller than dd_plan_get_info().workspace_bytes");
  if ((uintptr_t)ws & (kAlign - 1)) return fail(DD_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(ws, 0, kWsHeaderBytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace header reset");

  const uint8_t* base = reinterpret_cast<const uint8_t*>(p->device_base);
  AttnArgs a = base_args(cfg, q, kv, scales, ws, (size_t)p->num_slots);
  a.pages = reinterpret_cast<const uint32_t*>(base + p->off_pages);
  a.qorder = reinterpret_cast<const int32_t*>(base + p->off_qorder);
  a.qlimit = p->causal ? reinterpret_cast<const int32_t*>(base + p->off_qlimit) : nullptr;
  // The tcgen05 kernel (wide shared nodes, compute-bound) runs on tc_ctas
  // SMs and the streaming kernel (narrow nodes, HBM-bound), launched after it
  // in the same stream as a programmatic dependent, starts at once on the
  // other SMs and takes each tcgen05 CTA's SM when that CTA finishes; it
  // completes only after the tcgen05 grid, so the merge sees both. While
  // per-launch timing is on (dd_profile_enable), launches run one after the
  // other so each event pair brackets one kernel.
  const int n_tc = (int)p->items[kItemTc].size();
  const int n_tc2 = (int)p->items[kItemTc2].size();
  if (n_tc2) {
    a.items = reinterpret_cast<const WorkItem*>(base + p->off_items[kItemTc2]);
    rc = launch_attn_tc2(a, cfg->num_pages, n_tc2, st);
    if (rc) return rc;
  }
  if (n_tc) {
    a.items = reinterpret_cast<const WorkItem*>(base + p->off_items[kItemTc]);
    int grid = n_tc;
    if (p->tc_ctas > 0) {
      // A fixed number of CTAs, each running its scheduled items in turn.
      a.tc_order = reinterpret_cast<const int32_t*>(base + p->off_tc_order);
      a.tc_cta_begin = reinterpret_cast<const int32_t*>(base + p->off_tc_cta_begin);
      grid = p->tc_ctas;
    }
    rc = launch_attn_tc(a, cfg->num_pages, grid, st);
    a.tc_order = a.tc_cta_begin = nullptr;
    if (rc) return rc;
  }
  for (int k = 0; k < kNumItemKinds; ++k) {
    const int n = (int)p->items[k].size();
    if (!n || k == kItemTc || k == kItemTc2) continue;
    a.items = reinterpret_cast<const WorkItem*>(base + p->off_items[k]);
    if (k == kItemSimple) {
      e = launch_attn_simple(a, dim3(n), st);
      if (e != cudaSuccess) return cuda_fail(e, "attn_simple launch");
    } else {
      a.num_items = n;
      rc = launch_attn_mma(a, cfg->num_pages, st, n_tc > 0 && !prof_timing_on());
      if (rc) return rc;
    }
  }
  MergeArgs m;
  m.part_o = a.part_o;
  m.part_lse = a.part_lse;
  m.path_indptr = reinterpret_cast<const int32_t*>(base + p->off_pindptr);
  m.path_slots = reinterpret_cast<const int32_t*>(base + p->off_pslots);
  m.nsplit = 0;
  m.qorder = a.qorder;
  m.out = out;
  m.lse = lse;
  m.batch = p->batch_size;
  m.Hq = cfg->num_qo_heads;
  m.D = cfg->head_dim;
  m.out_dtype = cfg->q_dtype;
  if (po) {
    m.peer_out = po->ptrs;
    m.world = po->world;
    m.rank = po->rank;
    m.Hq_global = po->Hq_global;
    m.Hkv_global = po->Hkv_global;
    m.gqa_map = cfg->gqa_map;
  }
  e = launch_merge(m, st);
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return DD_OK;
}

extern "C" size_t dd_decode_paged_workspace_size(const dd_attn_config* cfg, int32_t B,
                                                 int32_t max_pages) {
  if (check_config(cfg) || B < 0 || max_pages < 0) return 0;
  const size_t ns = (size_t)flat_nsplit(cfg, B, max_pages);
  const size_t slots = ns * (size_t)B * cfg->num_qo_heads;
  return kWsHeaderBytes + align_up(slots * cfg->head_dim * sizeof(float), kAlign) +
         align_up(slots * sizeof(float), kAlign);
}

extern "C" int dd_decode_paged(const dd_attn_config* cfg, int32_t B, int32_t max_pages,
                               const void* q, const void* kv, const void* scales,
                               const int32_t* page_indptr, const int32_t* page_indices,
                               const int32_t* num_tokens, void* out, float* lse, void* ws,
                               size_t ws_bytes, dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (B < 0 || max_pages < 0) return fail(DD_ERR_INVALID_ARGUMENT, "bad batch size / max pages");
  if (B > 65535) return fail(DD_ERR_INVALID_ARGUMENT, "batch_size > 65535: use a plan (dd_cascade_decode)");
  if (B == 0) return DD_OK;
  if (!page_indptr || !num_tokens || (!page_indices && max_pages > 0))
    return fail(DD_ERR_INVALID_ARGUMENT, "page table pointer is NULL");
  rc = check_kv_ptrs(cfg, q, kv, scales, out);
  if (rc) return rc;
  const size_t need = dd_decode_paged_workspace_size(cfg, B, max_pages);
  if (!ws || ws_bytes < need) return fail(DD_ERR_WORKSPACE, "workspace smaller than dd_decode_paged_workspace_size");
  if ((uintptr_t)ws & (kAlign - 1)) return fail(DD_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(ws, 0, kWsHeaderBytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace header reset");
  const int ns = flat_nsplit(cfg, B, max_pages);
  AttnArgs a = base_args(cfg, q, kv, scales, ws, (size_t)ns * B * cfg->num_qo_heads);
  a.pages = reinterpret_cast<const uint32_t*>(page_indices);
  a.page_indptr = page_indptr;
  a.num_tokens = num_tokens;
  a.batch = B;
  a.nsplit = ns;
  const bool mma = cfg->q_dtype == DD_DTYPE_BF16 && mma_supported(cfg->head_dim, cfg->kv_dtype);
  a.row_tiles = mma ? (a.g + 15) / 16 : (a.g + 63) / 64;
  const dim3 grid(ns, cfg->num_kv_heads * a.row_tiles, B);
  if (mma) {
    a.num_items = ns * cfg->num_kv_heads * a.row_tiles * B;
    rc = launch_attn_mma(a, cfg->num_pages, st, false);
    if (rc) return rc;
  } else {
    e = launch_attn_simple(a, grid, st);
    if (e != cudaSuccess) return cuda_fail(e, "attn_simple launch");
  }
  MergeArgs m;
  m.part_o = a.part_o;
  m.part_lse = a.part_lse;
  m.path_indptr = nullptr;
  m.path_slots = nullptr;
  m.nsplit = ns;
  m.qorder = nullptr;
  m.out = out;
  m.lse = lse;
  m.batch = B;
  m.Hq = cfg->num_qo_heads;
  m.D = cfg->head_dim;
  m.out_dtype = cfg->q_dtype;
  e = launch_merge(m, st);
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return DD_OK;
}

extern "C" int dd_workspace_status(const void* ws, dd_stream_t stream, uint32_t* code,
                                   uint32_t* aux) {
  if (!ws || !code) return fail(DD_ERR_INVALID_ARGUMENT, "NULL argument");
  uint32_t h[2] = {0, 0};
  cudaError_t e = cudaMemcpyAsync(h, ws, sizeof(h), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "workspace status read");
  *code = h[0];
  if (aux) *aux = h[1];
  return DD_OK;
}

// --------------------------------------------------------------- append_kv
namespace dd {
__global__ void append_kv_kernel(void* kv, int dtype, uint32_t page, int slot0, int t, int Hkv,
                                 int D, const void* k, const void* v) {
  const int64_t n = (int64_t)2 * Hkv * t * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int tt = (int)((i / D) % t);
    const int h = (int)((i / ((int64_t)D * t)) % Hkv);
    const int which = (int)(i / ((int64_t)D * t * Hkv));
    const size_t src = ((size_t)h * t + tt) * D + d;
    const size_t dst = ((((size_t)page * 2 + which) * Hkv + h) * kPageSize + slot0 + tt) * D + d;
    const void* s = which ? v : k;
    if (dtype == DD_DTYPE_F32)
      reinterpret_cast<float*>(kv)[dst] = reinterpret_cast<const float*>(s)[src];
    else
      reinterpret_cast<uint16_t*>(kv)[dst] = reinterpret_cast<const uint16_t*>(s)[src];
  }
}

// One 16-byte chunk per thread and step: rows of D elements are contiguous
// on both sides, so the head-shard reorder is a gather of 16-byte vectors.
__global__ void scatter_heads_kernel(int world, int B, int Hq, int Hkv, int D, int gqa_map,
                                     int dtype, const void* gathered, void* out) {
  const int Hq_r = Hq / world, Hkv_r = Hkv / world, g = Hq / Hkv;
  const int cpr = D * (dtype == DD_DTYPE_F32 ? 4 : 2) / 16;  // chunks per row
  const int64_t rows = (int64_t)world * B * Hq_r;
  const int64_t n = rows * cpr;
  const uint4* src = reinterpret_cast<const uint4*>(gathered);
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / cpr;
    const int c = (int)(i - row * cpr);
    const int li = (int)(row % Hq_r);
    const int64_t rb = row / Hq_r;
    const int b = (int)(rb % B);
    const int r = (int)(rb / B);
    const int k0 = r * Hkv_r;
    // Local head li of rank r -> global query head (same GQA layout locally).
    const int h = gqa_map == DD_GQA_TILED ? (k0 + li % Hkv_r) + (li / Hkv_r) * Hkv : k0 * g + li;
    dst[((int64_t)b * Hq + h) * cpr + c] = src[i];
  }
}
}  // namespace dd

extern "C" int dd_append_kv(const dd_attn_config* cfg, void* kv, uint32_t block_id,
                            int32_t position, int32_t t, const void* k, const void* v,
                            dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (cfg->kv_dtype != DD_DTYPE_F32 && cfg->kv_dtype != DD_DTYPE_BF16)
    return fail(DD_ERR_NOT_AVAILABLE, "append_kv writes F32 or BF16 pages (quantize separately)");
  if (!kv || !k || !v) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if ((int64_t)block_id >= cfg->num_pages) return fail(DD_ERR_INVALID_ARGUMENT, "invalid block id: " + std::to_string(block_id));
  if (position < 0 || t <= 0 || position % kPageSize + t > kPageSize)
    return fail(DD_ERR_INVALID_ARGUMENT, "tokens must fit in the block at position % 16");
  const int64_t n = (int64_t)2 * cfg->num_kv_heads * t * cfg->head_dim;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 1024);
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  append_kv_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(kv, cfg->kv_dtype, block_id,
                                                             position % kPageSize, t,
                                                             cfg->num_kv_heads, cfg->head_dim, k, v);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "append_kv launch");
  return DD_OK;
}

extern "C" int dd_scatter_head_shards(const dd_attn_config* cfg, int32_t world, int32_t B,
                                      const void* gathered, void* out, dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (world <= 0 || cfg->num_kv_heads % world)
    return fail(DD_ERR_INVALID_ARGUMENT, "num_kv_heads must be divisible by world");
  if (B < 0) return fail(DD_ERR_INVALID_ARGUMENT, "bad batch size");
  if (B == 0) return DD_OK;
  if (!gathered || !out) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (((uintptr_t)gathered & 15) || ((uintptr_t)out & 15))
    return fail(DD_ERR_INVALID_ARGUMENT, "gathered / out must be 16-byte aligned");
  const int64_t n = (int64_t)B * cfg->num_qo_heads * cfg->head_dim * (cfg->q_dtype == DD_DTYPE_F32 ? 4 : 2) / 16;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  scatter_heads_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      world, B, cfg->num_qo_heads, cfg->num_kv_heads, cfg->head_dim, cfg->gqa_map, cfg->q_dtype,
      gathered, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "scatter_head_shards launch");
  return DD_OK;
}
