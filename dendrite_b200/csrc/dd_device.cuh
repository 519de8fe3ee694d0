// Device helpers shared by the sm_100a kernels: dtype conversions, mbarrier
// and TMA wrappers (inline PTX), bounded waits with an error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <climits>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dd_internal.h"
#include "dd_profile.h"

namespace dd {

// ---------------------------------------------------------------- error words
// The first 256 bytes of every workspace hold device-side status words.
enum DeviceError : uint32_t {
  kDevErrNone = 0,
  kDevErrBadPage = 1,      // page id >= num_pages in a device-side table
  kDevErrWaitTimeout = 2,  // an mbarrier wait exceeded its time limit
};
struct WsHeader {
  uint32_t error;      // first error code (DeviceError)
  uint32_t error_aux;     // e.g. offending page id
  uint32_t work_counter;  // next work item of a persistent kernel (zeroed per call)
  uint32_t pad[61];
};
static_assert(sizeof(WsHeader) == kWsHeaderBytes, "workspace header");

__device__ __forceinline__ void report_error(WsHeader* h, uint32_t code, uint32_t aux) {
  if (h && atomicCAS(&h->error, 0u, code) == 0u) h->error_aux = aux;
}

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float((uint32_t)b << 16);
}

// FP8 E4M3 code -> f32 (exact; the hardware conversion goes through f16).
__device__ __forceinline__ float e4m3_to_float(uint8_t c) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)c, __NV_E4M3);
  return __half2float(__half(h));
}

// Two E4M3 codes (low byte first) -> two f32.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t c2) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)c2, __NV_E4M3);
  return __half22float2(__half2(h));
}

// f32 -> E4M3, round to nearest even, saturating to +-448 (NaN stays NaN).
__device__ __forceinline__ uint8_t float_to_e4m3_satrn(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
// Four of them packed little-endian (a in byte 0), two per conversion.
__device__ __forceinline__ uint32_t e4m3x4_satrn(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (lo & 0xffffu) | (hi << 16);
}
// E8M0 shared exponent byte -> 2^(c-127) as f32 (c = 0 gives 2^-127, a
// subnormal f32; c = 255 is NaN in the format and is never produced).
// Branch-free: y = c << 23; c = 0 gives max(0, 2^-127 bits), c = 255 gives
// 0x7f800000, to which the carry out of y + 2^23 adds the quiet-NaN bit.
__device__ __forceinline__ float e8m0_bits_to_float(uint32_t y) {
  return __uint_as_float(max(y, 0x00400000u) | (((y + 0x00800000u) >> 9) & 0x00400000u));
}
__device__ __forceinline__ float e8m0_to_float(uint8_t c) { return e8m0_bits_to_float((uint32_t)c << 23); }
// The same for the E8M0 byte `b` (0-3) of a word.
__device__ __forceinline__ float e8m0_byte_to_float(uint32_t w, uint32_t b) {
  return e8m0_bits_to_float(__byte_perm(w, 0u, 0x0444u | (b << 12)) >> 1);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed pair arithmetic (sm_100 f32x2 instructions: two lanes of f32 per
// instruction) and a three-input max, for the softmax inner loops.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return ((uint64_t)__float_as_uint(b) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 16 E4M3 codes -> 16 bf16 = code * mul (f32 product, rounded once to bf16;
// exact for E4M3 times a power of two in bf16's normal range). The hardware
// E4M3 -> f16 conversion keeps NaN codes NaN. An integer-only variant (codes
// placed into bf16 bits, then one bf16 multiply) measured slower on B200.
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Four E4M3 codes (bytes 0-3 of w) times mul to two bf16x2 words (bytes 0-1
// -> r0, 2-3 -> r1): hardware E4M3 -> f16 -> f32, one packed f32 product per
// pair, round to nearest even to bf16.
__device__ __forceinline__ void e4m3x4_to_bf16_cvt(uint32_t w, float mul, uint32_t& r0, uint32_t& r1) {
  const float2 a = e4m3x2_to_float2((uint16_t)(w & 0xffffu));
  const float2 b = e4m3x2_to_float2((uint16_t)(w >> 16));
  const uint64_t m2 = f2_pack(mul, mul);
  const uint64_t pa = f2_mul(f2_pack(a.x, a.y), m2), pb = f2_mul(f2_pack(b.x, b.y), m2);
  r0 = pack_bf16x2(f2_lo(pa), f2_hi(pa));
  r1 = pack_bf16x2(f2_lo(pb), f2_hi(pb));
}
// Four E4M3 codes (bytes 0-3 of w), each with its own multiplier, to two
// bf16x2 words (bytes 0-1 -> r0, 2-3 -> r1); same rounding as above.
__device__ __forceinline__ void e4m3x4_to_bf16_mul4(uint32_t w, const float (&m)[4], uint32_t& r0,
                                                    uint32_t& r1) {
  const float2 a = e4m3x2_to_float2((uint16_t)(w & 0xffffu));
  const float2 b = e4m3x2_to_float2((uint16_t)(w >> 16));
  const uint64_t pa = f2_mul(f2_pack(a.x, a.y), f2_pack(m[0], m[1]));
  const uint64_t pb = f2_mul(f2_pack(b.x, b.y), f2_pack(m[2], m[3]));
  r0 = pack_bf16x2(f2_lo(pa), f2_hi(pa));
  r1 = pack_bf16x2(f2_lo(pb), f2_hi(pb));
}
__device__ __forceinline__ void e4m3x16_to_bf16(const uint4 c, float mul, uint32_t (&r)[8]) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) e4m3x4_to_bf16_cvt(w[i], mul, r[2 * i], r[2 * i + 1]);
}

// Two-term bf16 split of a pair of non-negative finite floats (softmax
// probabilities): x = hi + lo + e with hi = x truncated to bf16, lo = (x - hi)
// truncated to bf16 (x - hi is exact in f32). |e| < 2^-14 |x|. Only integer
// and f32 add units are used (no conversion instructions), so the split costs
// nothing on the pipe that also evaluates the exponentials.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  hi = __byte_perm(ua, ub, 0x7632);  // high halves: a in the low 16 bits
  const float ra = a - __uint_as_float(ua & 0xffff0000u);
  const float rb = b - __uint_as_float(ub & 0xffff0000u);
  lo = __byte_perm(__float_as_uint(ra), __float_as_uint(rb), 0x7632);
}

// split_bf16x2 with the two subtractions as one packed instruction.
__device__ __forceinline__ void split_bf16x2_packed(uint64_t ab, uint32_t& hi, uint32_t& lo) {
  const uint32_t ua = (uint32_t)ab, ub = (uint32_t)(ab >> 32);
  hi = __byte_perm(ua, ub, 0x7632);
  const uint64_t r = f2_sub(ab, ((uint64_t)(ub & 0xffff0000u) << 32) | (ua & 0xffff0000u));
  lo = __byte_perm((uint32_t)r, (uint32_t)(r >> 32), 0x7632);
}

// ------------------------------------------------------------------- timing
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legal wait

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and sets *abort, and the workspace error
// word) if the phase does not complete within limit_ns, or immediately if
// *abort is already set.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                WsHeader* err, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort = 1;
        report_error(err, kDevErrWaitTimeout, 0);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          WsHeader* err) {
  return mbar_wait_limit(bar, parity, abort, err, kWaitLimitNs);
}

// ----------------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load global -> shared, completion on an mbarrier.
// The innermost coordinate x is always 0 or a multiple of 64 elements here.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// The same two copies with an L2 cache-eviction policy (from l2_policy).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int32_t x,
                                                 int32_t y, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// L2 policies: evict_first for data this CTA alone reads once (a streamed
// leaf's pages), so it does not push out what other CTAs or the next kernel
// re-read (shared prefix pages, partial states); evict_normal otherwise.
__device__ __forceinline__ uint64_t l2_policy(bool evict_first) {
  uint64_t pol;
  if (evict_first)
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  else
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Named barrier among `nthreads` threads (multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------- math
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Query head served by row j (0..g-1) of KV head k.
__device__ __forceinline__ int qo_head_of(int gqa_map, int kv_head, int j, int Hkv, int g) {
  return gqa_map == DD_GQA_TILED ? kv_head + j * Hkv : kv_head * g + j;
}

// Device description of where an item's rows read queries and write partial
// states (shared by the attention kernels).
struct AttnArgs {
  const void* q;           // [B][Hq][D] bf16 or f32
  const void* kv;          // page pool
  const void* scales;      // per-head f32[2][Hkv] or E8M0 bytes
  float* part_o;           // [slots][D]
  float* part_lse;         // [slots], log2 domain
  WsHeader* err;
  const uint32_t* pages;   // plan page list (cascade) / page_indices (flat)
  const int32_t* qorder;   // DFS position -> query (NULL: identity)
  const WorkItem* items;   // cascade items (NULL: flat mode)
  // Causal (prefill) plans: tokens of its node (from the node's first token,
  // where every item starts) visible to each DFS query; NULL: all of them.
  const int32_t* qlimit;
  // tcgen05 items scheduled onto a fixed number of CTAs: CTA c runs items
  // tc_order[tc_cta_begin[c] .. tc_cta_begin[c + 1]) in turn (NULL: one item
  // per CTA, item blockIdx.x).
  const int32_t* tc_order;
  const int32_t* tc_cta_begin;
  // flat mode
  const int32_t* page_indptr;
  const int32_t* num_tokens;
  int32_t batch, nsplit, row_tiles;
  int32_t num_items;       // work items of this launch (persistent kernels)
  // config
  int32_t Hq, Hkv, g, D, kv_dtype, q_dtype, gqa_map, num_pages;
  float scale_log2;        // softmax scale * log2(e)
};

// Resolve this CTA's work item. In flat mode the grid is
// (nsplit, Hkv * row_tiles, batch) and each CTA takes a contiguous page range.
__device__ __forceinline__ WorkItem resolve_item(const AttnArgs& a, const uint32_t*& pages,
                                                 int row_tile_rows) {
  WorkItem it;
  if (a.items) {
    it = a.items[blockIdx.x];
    pages = a.pages + it.page_off;
    return it;
  }
  const int s = blockIdx.x, b = blockIdx.z;
  const int h = blockIdx.y / a.row_tiles, t = blockIdx.y % a.row_tiles;
  const int ntok = a.num_tokens[b];
  const int P = (ntok + kPageSize - 1) / kPageSize;
  const int pb = (int)((int64_t)s * P / a.nsplit), pe = (int)((int64_t)(s + 1) * P / a.nsplit);
  it.page_off = 0;
  it.npages = pe - pb;
  it.last_valid = (pe == P && (ntok % kPageSize)) ? ntok % kPageSize : kPageSize;
  it.kv_head = h;
  it.row0 = t * row_tile_rows;
  it.nrows = min(row_tile_rows, a.g - it.row0);
  it.q_begin = b;
  it.slot_base = (s * a.batch + b) * a.Hq;
  pages = a.pages + a.page_indptr[b] + pb;
  return it;
}

// Same, for persistent kernels: work item `idx` of `a.num_items`. Flat mode
// enumerates (split, KV head x row tile, query) with the split fastest.
__device__ __forceinline__ WorkItem resolve_item_idx(const AttnArgs& a, int idx,
                                                     const uint32_t*& pages, int row_tile_rows) {
  WorkItem it;
  if (a.items) {
    it = a.items[idx];
    pages = a.pages + it.page_off;
    return it;  // nrows may carry kItemSoleReader: callers mask with kItemRowsMask
  }
  const int s = idx % a.nsplit;
  const int rest = idx / a.nsplit;
  const int y = rest % (a.Hkv * a.row_tiles), b = rest / (a.Hkv * a.row_tiles);
  const int h = y / a.row_tiles, t = y % a.row_tiles;
  const int ntok = a.num_tokens[b];
  const int P = (ntok + kPageSize - 1) / kPageSize;
  const int pb = (int)((int64_t)s * P / a.nsplit), pe = (int)((int64_t)(s + 1) * P / a.nsplit);
  it.page_off = 0;
  it.npages = pe - pb;
  it.last_valid = (pe == P && (ntok % kPageSize)) ? ntok % kPageSize : kPageSize;
  it.kv_head = h;
  it.row0 = t * row_tile_rows;
  it.nrows = min(row_tile_rows, a.g - it.row0);
  it.q_begin = b;
  it.slot_base = (s * a.batch + b) * a.Hq;
  pages = a.pages + a.page_indptr[b] + pb;
  return it;
}

// Inputs of the path merge (merge.cu). Path source: CSR (cascade plans) or
// strided (flat split-K decode: slot (s * batch + p) * Hq for s < nsplit).
struct MergeArgs {
  const float* part_o;
  const float* part_lse;
  const int32_t* path_indptr;
  const int32_t* path_slots;
  int32_t nsplit;
  const int32_t* qorder;
  void* out;
  float* lse;
  int32_t batch, Hq, D, out_dtype;
  // Head-split decode with the outputs written straight into every rank's
  // output buffer (peer memory): peer_out[world] device pointers to
  // [batch][Hq_global][D]; this rank's local head h goes to its global head.
  void* const* peer_out = nullptr;
  int32_t world = 1, rank = 0, Hq_global = 0, Hkv_global = 0, gqa_map = 0;
};

}  // namespace dd
