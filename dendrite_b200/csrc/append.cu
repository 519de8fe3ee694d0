// Decode-step KV writes into the page pool: a batched append with the FP8
// quantization fused in, and the page copy of copy-on-write.
//
// ReferenceBackend::append_kv (crates/dendrite-core/src/attention/backend.rs:285-301)
// stores one sequence's tokens per call, and BlockPool::copy_on_write
// (crates/dendrite-core/src/cache/pool.rs:88-91) swaps the block id without
// copying data. A decode step of an engine appends one token to every
// sequence; here that is one launch over device arrays of (page, slot)
// targets, writing the pool's storage type directly:
//   F32 / BF16 pages   the values (bf16 round-to-nearest-even from f32);
//   E4M3 pages         RNE-saturating E4M3 of x / scale[kv][h], the pool's
//                      per-head scales (the codes dd_quantize_kv_pages writes
//                      for these values under those scales);
//   MXFP8 pages        per 32-element block of the token's head vector, the
//                      E8M0 exponent and codes dd_quantize_kv_pages writes
//                      (OCP MX: e = max(-127, floor(log2 amax) - 8)).
// dd_copy_pages gives copy-on-write its data copy: whole pages, codes and
// MXFP8 exponents included.
#include "dd_device.cuh"

namespace dd {

__device__ __forceinline__ int floor_log2_pos(float a) {
  const uint32_t b = __float_as_uint(a);
  const int e = (int)((b >> 23) & 0xff);
  if (e != 0) return e - 127;
  return (31 - __clz((int)(b & 0x7fffff))) - 149;
}

// One warp per (token, K/V, head); lane owns E = D/32 consecutive elements.
template <int D>
__global__ void append_batch_kernel(int32_t n, int Hkv, int num_pages, int pool_dtype, int src_dtype,
                                    void* kv, void* scales, const uint32_t* page_ids,
                                    const int32_t* slots, const void* k, const void* v,
                                    uint32_t* status) {
  constexpr int E = D / 32;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (int64_t)n * 2 * Hkv) return;
  const int h = (int)(warp % Hkv);
  const int which = (int)((warp / Hkv) % 2);
  const int32_t tok = (int32_t)(warp / (2 * Hkv));
  const uint32_t page = page_ids[tok];
  const int32_t slot = slots[tok];
  if (page >= (uint32_t)num_pages || slot < 0 || slot >= kPageSize) {
    if (lane == 0 && status && atomicCAS(status, 0u, 1u) == 0u) status[1] = (uint32_t)tok;
    return;
  }
  // Source row [tok][h][D], this lane's E elements.
  const size_t src_off = ((size_t)tok * Hkv + h) * D + lane * E;
  const void* src = which ? v : k;
  float x[E];
  if (src_dtype == DD_DTYPE_F32) {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = reinterpret_cast<const float*>(src)[src_off + e];
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e)
      x[e] = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(src)[src_off + e] << 16);
  }
  const int64_t row = ((int64_t)page * 2 + which) * Hkv + h;   // (page, K/V, head) slice
  const size_t dst_off = ((size_t)row * kPageSize + slot) * D + lane * E;
  if (pool_dtype == DD_DTYPE_F32) {
#pragma unroll
    for (int e = 0; e < E; ++e) reinterpret_cast<float*>(kv)[dst_off + e] = x[e];
  } else if (pool_dtype == DD_DTYPE_BF16) {
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(kv) + dst_off + e) = pack_bf16x2(x[e], x[e + 1]);
  } else if (pool_dtype == DD_DTYPE_E4M3) {
    const float sc = reinterpret_cast<const float*>(scales)[which * Hkv + h];
#pragma unroll
    for (int e = 0; e < E; ++e)
      reinterpret_cast<uint8_t*>(kv)[dst_off + e] = float_to_e4m3_satrn(__fdiv_rn(x[e], sc));
  } else {
    // MXFP8: the 32 / E lanes of a block agree on its amax.
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) m = fmaxf(m, fabsf(x[e]));
#pragma unroll
    for (int o = 1; o < 32 / E; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int ex = m > 0.f ? floor_log2_pos(m) - 8 : -127;
    if (ex < -127) ex = -127;
    const float inv = __uint_as_float((uint32_t)(127 - ex) << 23);  // 2^-ex, a normal f32
#pragma unroll
    for (int e = 0; e < E; ++e)
      reinterpret_cast<uint8_t*>(kv)[dst_off + e] = float_to_e4m3_satrn(x[e] * inv);
    if ((lane * E) % 32 == 0)
      reinterpret_cast<uint8_t*>(scales)[((size_t)row * kPageSize + slot) * (D / 32) + (lane * E) / 32] =
          (uint8_t)(ex + 127);
  }
}

// One CTA per (source, destination) page pair; 16-byte copies of the page's
// K/V data and, for MXFP8, its exponent bytes.
__global__ void copy_pages_kernel(int32_t n, int num_pages, size_t page_bytes, size_t scale_bytes,
                                  uint8_t* kv, uint8_t* scales, const uint32_t* src,
                                  const uint32_t* dst, uint32_t* status) {
  const int32_t i = blockIdx.x;
  if (i >= n) return;
  const uint32_t s = src[i], d = dst[i];
  if (s >= (uint32_t)num_pages || d >= (uint32_t)num_pages) {
    if (threadIdx.x == 0 && status && atomicCAS(status, 0u, 2u) == 0u) status[1] = (uint32_t)i;
    return;
  }
  if (s == d) return;
  const uint4* a = reinterpret_cast<const uint4*>(kv + (size_t)s * page_bytes);
  uint4* b = reinterpret_cast<uint4*>(kv + (size_t)d * page_bytes);
  for (size_t j = threadIdx.x; j < page_bytes / 16; j += blockDim.x) b[j] = a[j];
  if (scale_bytes) {
    const uint8_t* sa = scales + (size_t)s * scale_bytes;
    uint8_t* sb = scales + (size_t)d * scale_bytes;
    for (size_t j = threadIdx.x; j < scale_bytes; j += blockDim.x) sb[j] = sa[j];
  }
}

// The kernels' bounded wait, run out on purpose: an mbarrier that nothing
// arrives on, waited for with limit_ns; the wait gives up, records
// kDevErrWaitTimeout in the workspace header and the kernel returns.
__global__ void selftest_wait_kernel(WsHeader* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  mbar_init(&bar, 1);
  abort = 0;
  fence_mbar_init();
  mbar_wait_limit(&bar, 0, &abort, err, limit_ns);
}

}  // namespace dd

using namespace dd;

extern "C" int dd_selftest_wait(void* workspace, uint64_t limit_ns, dd_stream_t stream) {
  if (!workspace) return fail(DD_ERR_INVALID_ARGUMENT, "workspace is NULL");
  if (limit_ns == 0 || limit_ns > kWaitLimitNs) return fail(DD_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 2 s]");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(workspace, 0, kWsHeaderBytes, st);
  if (e == cudaSuccess) {
    selftest_wait_kernel<<<1, 1, 0, st>>>(reinterpret_cast<WsHeader*>(workspace), limit_ns);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("selftest_wait: ") + cudaGetErrorString(e));
  return DD_OK;
}

extern "C" int dd_append_kv_batch(const dd_attn_config* cfg, void* kv_pages, void* kv_scales,
                                  int32_t n, const uint32_t* page_ids, const int32_t* slots,
                                  const void* k, const void* v, int32_t src_dtype,
                                  uint32_t* status, dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (n < 0) return fail(DD_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (n == 0) return DD_OK;
  if (!kv_pages || !page_ids || !slots || !k || !v)
    return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (src_dtype != DD_DTYPE_F32 && src_dtype != DD_DTYPE_BF16)
    return fail(DD_ERR_INVALID_ARGUMENT, "source K/V must be f32 or bf16");
  const bool fp8 = cfg->kv_dtype == DD_DTYPE_E4M3 || cfg->kv_dtype == DD_DTYPE_MXFP8;
  if (fp8 && !kv_scales) return fail(DD_ERR_INVALID_ARGUMENT, "FP8 pages need kv_scales");
  const int64_t warps = (int64_t)n * 2 * cfg->num_kv_heads;
  const int blocks = (int)((warps * 32 + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(kProfOther, st);
  switch (cfg->head_dim) {
#define DD_APPEND(DIM)                                                                          \
  case DIM:                                                                                     \
    append_batch_kernel<DIM><<<blocks, 256, 0, st>>>(n, cfg->num_kv_heads, cfg->num_pages,     \
                                                     cfg->kv_dtype, src_dtype, kv_pages,       \
                                                     kv_scales, page_ids, slots, k, v, status); \
    break;
    DD_APPEND(64)
    DD_APPEND(128)
    DD_APPEND(256)
#undef DD_APPEND
    default:
      return fail(DD_ERR_INVALID_ARGUMENT, "unsupported head_dim");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("append_kv_batch launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

extern "C" int dd_copy_pages(const dd_attn_config* cfg, void* kv_pages, void* kv_scales, int32_t n,
                             const uint32_t* src, const uint32_t* dst, uint32_t* status,
                             dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (n < 0) return fail(DD_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (n == 0) return DD_OK;
  if (!kv_pages || !src || !dst) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (((uintptr_t)kv_pages & 15) != 0) return fail(DD_ERR_INVALID_ARGUMENT, "kv_pages not 16-byte aligned");
  const size_t elem = cfg->kv_dtype == DD_DTYPE_F32 ? 4 : cfg->kv_dtype == DD_DTYPE_BF16 ? 2 : 1;
  const size_t page_bytes = (size_t)2 * cfg->num_kv_heads * kPageSize * cfg->head_dim * elem;
  size_t scale_bytes = 0;
  if (cfg->kv_dtype == DD_DTYPE_MXFP8) {
    if (!kv_scales) return fail(DD_ERR_INVALID_ARGUMENT, "MXFP8 pages need kv_scales");
    scale_bytes = (size_t)2 * cfg->num_kv_heads * kPageSize * (cfg->head_dim / 32);
  }
  cudaStream_t st = (cudaStream_t)stream;
  {
    ProfScope ps(kProfOther, st);
    copy_pages_kernel<<<n, 256, 0, st>>>(n, cfg->num_pages, page_bytes, scale_bytes,
                                         reinterpret_cast<uint8_t*>(kv_pages),
                                         reinterpret_cast<uint8_t*>(kv_scales), src, dst, status);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("copy_pages launch: ") + cudaGetErrorString(e));
  return DD_OK;
}
