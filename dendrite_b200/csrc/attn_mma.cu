// Paged partial attention for cascade nodes with up to 64 query rows per KV
// head (leaves, deep shared nodes, flat batch decode), bf16 / E4M3 / MXFP8 KV.
//
// Structure (one CTA per work item, 4 consumer warps + 1 producer warp):
//  - the producer lane streams the item's pages through a ring of shared
//    memory stages with TMA (cp.async.bulk.tensor, 128-byte swizzle) — four
//    16-token pages of K and V per stage, each page slice [16][head_dim]
//    contiguous in the pool — completion tracked by mbarriers;
//  - FP8 pages land as 1-byte codes (+ E8M0 bytes for MXFP8) and the consumer
//    warps dequantise them to bf16 in shared memory (code * scale, rounded to
//    bf16), so the HBM stream stays 1 byte per element;
//  - each consumer warp owns 16 query rows (a GQA group of one or more
//    queries that share the node) and a subset of the stage's pages, runs
//    q.k^T and p.v as m16n8k16 bf16 tensor-core tiles with f32 accumulators,
//    and keeps an online softmax (running max / sum in the log2 domain);
//  - warps that split the pages of a node combine their states through shared
//    memory; the CTA writes one normalised partial state per row.
// The arithmetic is ReferenceBackend::decode's
// (crates/dendrite-core/src/attention/backend.rs:254-262) over the node's
// tokens; partial states are merged by merge.cu along each query's path.
#include "dd_device.cuh"

namespace dd {

constexpr int kMmaRows = 64;       // rows per item (4 warps x 16)
constexpr int kMmaConsumers = 4;   // consumer warps
constexpr int kMmaThreads = (kMmaConsumers + 1) * 32;
constexpr int kStagePages = 4;

enum KvKind { kKvBf16 = 0, kKvE4m3 = 1, kKvMx = 2 };

template <int D, int KV>
struct MmaCfg {
  static constexpr int kSliceBf16 = kPageSize * D * 2;                 // one page, K or V
  static constexpr int kSliceRaw = KV == kKvBf16 ? kSliceBf16 : kPageSize * D;
  static constexpr int kMxBytes = KV == kKvMx ? kPageSize * (D / 32) : 0;
  static constexpr int kStages = KV == kKvBf16 ? (D == 128 ? 3 : 4) : 4;
  static constexpr int kRawStage = 2 * kStagePages * kSliceRaw;        // K pages then V pages
  static constexpr int kMxStage = 2 * kStagePages * kMxBytes;
  static constexpr int kRawStageAll = kRawStage + (kMxStage ? ((kMxStage + 1023) / 1024) * 1024 : 0);
  static constexpr int kConvBytes = KV == kKvBf16 ? 0 : 2 * kStagePages * kSliceBf16;
  static constexpr int kCombineBytes = kMmaConsumers * 16 * D * 4 + 2 * kMmaConsumers * 16 * 4;
  static constexpr int kPipeBytes = kStages * kRawStageAll + kConvBytes;
  static constexpr int kSmemBytes =
      (kPipeBytes > kCombineBytes ? kPipeBytes : kCombineBytes) + 1024;  // + alignment slack
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` (8 bf16 along D) of token row `t`
// inside a bf16 page slice stored as D/64 TMA boxes of [16][128 B] with the
// 128-byte swizzle (chunk index XOR row % 8).
__device__ __forceinline__ uint32_t swz_bf16(int t, int chunk) {
  return (uint32_t)((chunk >> 3) * 2048 + t * 128 + (((chunk & 7) ^ (t & 7)) << 4));
}

template <int D, int KV>
__global__ void __launch_bounds__(kMmaThreads)
    attn_mma_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a) {
  using C = MmaCfg<D, KV>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ int abort_flag;
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* conv = smem + S * C::kRawStageAll;

  const uint32_t* pages;
  const WorkItem it = resolve_item(a, pages, kMmaRows);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npages = it.npages;
  const int nst = (npages + kStagePages - 1) / kStagePages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kMmaConsumers);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x == kMmaConsumers * 32) prefetch_tmap(&kv_map);
  __syncthreads();

  if (warp == kMmaConsumers) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(&empty_bar[s], ((i / S) - 1) & 1, &abort_flag, a.err)) break;
        const int np = min(kStagePages, npages - i * kStagePages);
        const uint32_t bytes = (uint32_t)np * 2 * (C::kSliceRaw + C::kMxBytes);
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        uint8_t* st = smem + s * C::kRawStageAll;
        for (int j = 0; j < np; ++j) {
          uint32_t page = pages[i * kStagePages + j];
          if (page >= (uint32_t)a.num_pages) {
            report_error(a.err, kDevErrBadPage, page);
            page = 0;  // load something harmless; consumers mask the page
          }
          for (int kv = 0; kv < 2; ++kv) {
            const int y = (int)((((int64_t)page * 2 + kv) * a.Hkv + it.kv_head) * kPageSize);
            uint8_t* dst = st + (kv * kStagePages + j) * C::kSliceRaw;
            if (KV == kKvBf16) {
#pragma unroll
              for (int hb = 0; hb < D / 64; ++hb)
                tma_load_2d(dst + hb * 2048, &kv_map, hb * 64, y, &full_bar[s]);
            } else {
              tma_load_2d(dst, &kv_map, 0, y, &full_bar[s]);
              if (KV == kKvMx) {
                const uint8_t* src = reinterpret_cast<const uint8_t*>(a.scales) +
                                     (size_t)y * (D / 32);
                bulk_load(st + C::kRawStage + (kv * kStagePages + j) * C::kMxBytes, src,
                          C::kMxBytes, &full_bar[s]);
              }
            }
          }
        }
      }
    }
    // fall through to the final CTA barrier
  } else {
    // ------------------------------------------------------------ consumers
    const int nrows = it.nrows;
    int RG = (nrows + 15) / 16;
    if (RG == 3) RG = 4;
    const int TG = kMmaConsumers / RG;
    const int rg = warp / TG, tg = warp % TG;
    const int ctid = threadIdx.x;  // 0..127

    // Query fragments (A operand, rows rg*16 + lane/4 and +8).
    uint32_t qa[D / 16][4];
    {
      const int r0 = rg * 16 + (lane >> 2);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = r0 + half * 8;
        const uint32_t* qrow = nullptr;
        if (r < nrows) {
          const int rr = it.row0 + r, qi = rr / a.g;
          const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
          const int qid = a.qorder ? a.qorder[it.q_begin + qi] : it.q_begin + qi;
          qrow = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint16_t*>(a.q) +
                                                   ((size_t)qid * a.Hq + hq) * D);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk * 8 + (lane & 3);  // u32 index of (kk*16 + (lane%4)*2)
          qa[kk][half] = qrow ? qrow[c] : 0u;
          qa[kk][2 + half] = qrow ? qrow[c + 4] : 0u;
        }
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    float sc_k = 1.f, sc_v = 1.f;
    if (KV == kKvE4m3) {
      sc_k = reinterpret_cast<const float*>(a.scales)[it.kv_head];
      sc_v = reinterpret_cast<const float*>(a.scales)[a.Hkv + it.kv_head];
    }

    for (int i = 0; i < nst; ++i) {
      const int s = i % S;
      const bool ok = mbar_wait(&full_bar[s], (i / S) & 1, &abort_flag, a.err);
      const int np = min(kStagePages, npages - i * kStagePages);
      const uint8_t* kbase;
      const uint8_t* vbase;
      const uint8_t* st = smem + s * C::kRawStageAll;
      if (KV == kKvBf16) {
        kbase = st;
        vbase = st + kStagePages * C::kSliceRaw;
      } else {
        // Dequantise the stage into the bf16 buffer: wait until every
        // consumer is done with the previous contents first.
        named_bar_sync(1, kMmaConsumers * 32);
        if (ok) {
          for (int u = ctid; u < np * 2 * kPageSize * (D / 16); u += kMmaConsumers * 32) {
            const int c = u % (D / 16);            // 16-code chunk along D
            const int t = (u / (D / 16)) % kPageSize;
            const int kv = (u / (D / 16 * kPageSize)) & 1;
            const int j = u / (D / 16 * kPageSize * 2);
            const uint8_t* src = st + (kv * kStagePages + j) * C::kSliceRaw + t * D +
                                 (((c & 7) ^ (t & 7)) << 4);
            const uint4 codes = *reinterpret_cast<const uint4*>(src);
            float sc;
            if (KV == kKvE4m3) {
              sc = kv ? sc_v : sc_k;
            } else {
              sc = e8m0_to_float(st[C::kRawStage + (kv * kStagePages + j) * C::kMxBytes +
                                    t * (D / 32) + (c >> 1)]);
            }
            const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
            uint32_t outw[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f0 = e4m3x2_to_float2((uint16_t)(w[q] & 0xffff));
              const float2 f1 = e4m3x2_to_float2((uint16_t)(w[q] >> 16));
              outw[2 * q] = pack_bf16x2(f0.x * sc, f0.y * sc);
              outw[2 * q + 1] = pack_bf16x2(f1.x * sc, f1.y * sc);
            }
            uint8_t* dst = conv + (kv * kStagePages + j) * C::kSliceBf16;
            *reinterpret_cast<uint4*>(dst + swz_bf16(t, 2 * c)) =
                make_uint4(outw[0], outw[1], outw[2], outw[3]);
            *reinterpret_cast<uint4*>(dst + swz_bf16(t, 2 * c + 1)) =
                make_uint4(outw[4], outw[5], outw[6], outw[7]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);  // raw stage may be refilled
        named_bar_sync(1, kMmaConsumers * 32);
        kbase = conv;
        vbase = conv + kStagePages * C::kSliceBf16;
      }
      if (ok) {
        for (int jj = tg; jj < np; jj += TG) {
          const int pi = i * kStagePages + jj;
          int valid = (pi == npages - 1) ? it.last_valid : kPageSize;
          if (pages[pi] >= (uint32_t)a.num_pages) valid = 0;
          if (valid == 0) continue;
          const uint32_t kaddr = smem_u32(kbase + jj * C::kSliceBf16);
          const uint32_t vaddr = smem_u32(vbase + jj * C::kSliceBf16);
          // S = Q K^T for 16 rows x 16 tokens.
          float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int t = ((lane >> 4) << 3) + (lane & 7);
            const int chunk = kk * 2 + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kaddr + swz_bf16(t, chunk), b0, b1, b2, b3);
            mma_bf16(s0, qa[kk], b0, b1);
            mma_bf16(s1, qa[kk], b2, b3);
          }
          // Scale, mask, online softmax (log2 domain).
          const int tc = (lane & 3) * 2;
          float x[8] = {s0[0], s0[1], s1[0], s1[1], s0[2], s0[3], s1[2], s1[3]};
          const int tok[4] = {tc, tc + 1, 8 + tc, 9 + tc};
#pragma unroll
          for (int e = 0; e < 8; ++e)
            x[e] = tok[e & 3] < valid ? x[e] * a.scale_log2 : -INFINITY;
          float mx0 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
          float mx1 = fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7]));
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
          const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
          const float al0 = fast_exp2(m0 - nm0), al1 = fast_exp2(m1 - nm1);
          m0 = nm0;
          m1 = nm1;
          float p[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) p[e] = fast_exp2(x[e] - nm0);
#pragma unroll
          for (int e = 4; e < 8; ++e) p[e] = fast_exp2(x[e] - nm1);
          l0 = l0 * al0 + (p[0] + p[1] + p[2] + p[3]);
          l1 = l1 * al1 + (p[4] + p[5] + p[6] + p[7]);
#pragma unroll
          for (int n = 0; n < D / 8; ++n) {
            o[n][0] *= al0;
            o[n][1] *= al0;
            o[n][2] *= al1;
            o[n][3] *= al1;
          }
          // P = P_hi + P_lo, both bf16: the two P.V products carry P to
          // ~16 significant bits, so rounding P costs no accuracy.
          uint32_t pa[4], pl[4];
          split_bf16x2(p[0], p[1], pa[0], pl[0]);
          split_bf16x2(p[4], p[5], pa[1], pl[1]);
          split_bf16x2(p[2], p[3], pa[2], pl[2]);
          split_bf16x2(p[6], p[7], pa[3], pl[3]);
          // O += P V.
#pragma unroll
          for (int nn = 0; nn < D / 16; ++nn) {
            const int t = (((lane >> 3) & 1) << 3) + (lane & 7);
            const int chunk = nn * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vaddr + swz_bf16(t, chunk), b0, b1, b2, b3);
            mma_bf16(o[2 * nn], pa, b0, b1);
            mma_bf16(o[2 * nn + 1], pa, b2, b3);
            mma_bf16(o[2 * nn], pl, b0, b1);
            mma_bf16(o[2 * nn + 1], pl, b2, b3);
          }
        }
      }
      if (KV == kKvBf16) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
      }
    }

    // Row sums across the quad.
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // Stage every warp's state in shared memory (reusing the pipeline
    // buffers), then combine the page-split warps and write partial states.
    named_bar_sync(1, kMmaConsumers * 32);
    float* cmb_o = reinterpret_cast<float*>(smem);                     // [warp][16][D]
    float* cmb_m = cmb_o + kMmaConsumers * 16 * D;                     // [warp][16]
    float* cmb_l = cmb_m + kMmaConsumers * 16;
    {
      float* wo = cmb_o + warp * 16 * D;
      const int r = lane >> 2, c = (lane & 3) * 2;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        *reinterpret_cast<float2*>(wo + r * D + n * 8 + c) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2*>(wo + (r + 8) * D + n * 8 + c) = make_float2(o[n][2], o[n][3]);
      }
      if ((lane & 3) == 0) {
        cmb_m[warp * 16 + r] = m0;
        cmb_m[warp * 16 + r + 8] = m1;
        cmb_l[warp * 16 + r] = l0;
        cmb_l[warp * 16 + r + 8] = l1;
      }
    }
    named_bar_sync(1, kMmaConsumers * 32);
    for (int idx = ctid; idx < nrows * D; idx += kMmaConsumers * 32) {
      const int r = idx / D, d = idx % D;
      const int rgr = r >> 4, rl = r & 15;
      float M = -INFINITY;
      for (int t = 0; t < TG; ++t) M = fmaxf(M, cmb_m[(rgr * TG + t) * 16 + rl]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int t = 0; t < TG; ++t) {
          const int w = rgr * TG + t;
          const float f = fast_exp2(cmb_m[w * 16 + rl] - M);
          L += cmb_l[w * 16 + rl] * f;
          O += cmb_o[(w * 16 + rl) * D + d] * f;
        }
      }
      const int rr = it.row0 + r, qi = rr / a.g;
      const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
      const int64_t slot = (int64_t)it.slot_base + (int64_t)qi * a.Hq + hq;
      a.part_o[slot * D + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) a.part_lse[slot] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// 2-D view of the page pool: rows = num_pages * 2 * Hkv * 16 token rows of
// D elements; box = 16 rows x 128 bytes, 128-byte swizzle.
int make_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int Hkv, int D,
                       int elem_bytes) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const uint64_t rows = (uint64_t)num_pages * 2 * Hkv * kPageSize;
  if (rows == 0 || rows > 0x7FFFFFFFull)  // y coordinates are int32
    return fail(DD_ERR_INVALID_ARGUMENT, "page pool too large for a TMA descriptor");
  if (((uintptr_t)kv & 15) != 0) return fail(DD_ERR_INVALID_ARGUMENT, "kv_pages not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)kPageSize};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = enc(map, dt, 2, const_cast<void*>(kv), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DD_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return DD_OK;
}

template <int D, int KV>
static cudaError_t launch_mma_t(const CUtensorMap& map, const AttnArgs& a, dim3 grid,
                                cudaStream_t st) {
  const int smem = MmaCfg<D, KV>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<D, KV>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  {
    ProfScope ps(kProfMma, st);
    attn_mma_kernel<D, KV><<<grid, kMmaThreads, smem, st>>>(map, a);
  }
  return cudaGetLastError();
}

bool mma_supported(int D, int kv_dtype) {
  if (kv_dtype == DD_DTYPE_BF16) return D == 64 || D == 128;
  if (kv_dtype == DD_DTYPE_E4M3 || kv_dtype == DD_DTYPE_MXFP8) return D == 128;
  return false;
}

int launch_attn_mma(const AttnArgs& a, int64_t num_pages, dim3 grid, cudaStream_t st) {
  CUtensorMap map;
  const int eb = a.kv_dtype == DD_DTYPE_BF16 ? 2 : 1;
  int rc = make_kv_tensor_map(&map, a.kv, num_pages, a.Hkv, a.D, eb);
  if (rc) return rc;
  cudaError_t e;
  if (a.kv_dtype == DD_DTYPE_BF16)
    e = a.D == 64 ? launch_mma_t<64, kKvBf16>(map, a, grid, st)
                  : launch_mma_t<128, kKvBf16>(map, a, grid, st);
  else if (a.kv_dtype == DD_DTYPE_E4M3)
    e = launch_mma_t<128, kKvE4m3>(map, a, grid, st);
  else
    e = launch_mma_t<128, kKvMx>(map, a, grid, st);
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_mma launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

}  // namespace dd
