// tcgen05 partial attention on a CTA pair (two SMs, cta_group::2) for the
// widest shared nodes: items of up to 512 rows (> 256), bf16 pages and queries,
// head_dim 128.
//
// A cluster of two CTAs takes one work item = (node, KV head, 512-row tile,
// page range). CTA c (cluster rank) owns rows [256c, 256c + 256) as two
// 128-row sub-tiles A_c and B_c, and the pair multiplies with M = 256: one
// tcgen05.mma issued by the leader (rank 0) computes A_0 and A_1 (or B_0 and
// B_1) together, each CTA's 128 rows landing in its own TMEM. The B operand
// of an M = 256 product is split along N between the two CTAs, so each CTA
// loads only half of every tile:
//   K tile (S = Q.K^T, N = 128 tokens): CTA c holds tokens 64c..64c+63
//     (pages 4c..4c+3 of the tile) as [2 dim-halves][64 rows][128 B];
//   V tile (O += P.V, N = 128 dims):    CTA c holds dims 64c..64c+63 of all
//     128 tokens as [128 rows][128 B].
// Per SM that halves the K/V bytes moved and the B-operand shared-memory
// reads of the one-SM kernel (attn_tc.cu), which both bound it.
//
// Roles per CTA (320 threads), as in attn_tc.cu:
//   warp 0      producer: lanes 0-7 own the tile's 8 pages; K boxes of this
//               CTA's 4 pages, V boxes of its dim-half of all 8 pages, into a
//               ring of 16 KiB half-tiles. The copies use the CTA-pair form of
//               the TMA load, which completes on the leader's barrier, so the
//               leader sees both halves land on one barrier.
//   warp 1      TMEM (512 columns, allocated for the pair); in the leader,
//               lane 0 issues every product in the order
//               P_A.V_j, Q_A.K_{j+1}, P_B.V_j, Q_B.K_{j+1}
//               and commits each completion to both CTAs' barriers.
//   warps 2-9   softmax of this CTA's rows, one thread per row, written over
//               the scores as bf16 hi/lo terms (attn_tc.cu); arrivals that
//               release the leader's products go to the leader's barriers.
// Cross-CTA signals: mbarrier arrivals on the leader's barriers through
// mapa addresses (release.cluster) and waits with acquire.cluster; cluster
// barriers after setup and before teardown. Every wait is bounded.
#include "tc_common.cuh"

namespace dd {

constexpr int kT2Slots = 8;                   // ring of half-tiles
constexpr int kT2SlotBytes = 64 * 128 * 2;    // 16 KiB: 64 tokens x 128 dims, or 128 x 64
constexpr int kT2KHalf = 64 * 128;            // one 64-dim half of a K half-tile
constexpr int kT2Threads = 320;
constexpr int kT2Smem = 2 * kTcQBytes + kT2Slots * kT2SlotBytes + 1024;

// kind::f16, D f32, A/B bf16, M = 256 (pair), N = 128.
constexpr uint32_t kIdesc2QK = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) |
                               ((256u >> 4) << 24);
constexpr uint32_t kIdesc2PV = kIdesc2QK | (1u << 16);  // B (V) MN-major

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals may come from the peer).
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, volatile int* abort,
                                             WsHeader* err) {
  if (mbar_try_wait_cl(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        report_error(err, kDevErrWaitTimeout, 3);
        return false;
      }
    }
  }
}
// 2-D tiled load into this CTA's shared memory, completing on an mbarrier of
// either CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t x,
                                                 int32_t y, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma2_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma2_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
// Completion of the pair's prior products, signalled on the barrier at
// `bar` in both CTAs (one commit per CTA).
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   peer_addr(bar, 0))
               : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   peer_addr(bar, 1))
               : "memory");
}

struct Tc2Bars {
  uint64_t kv_full[kT2Slots];   // leader: both CTAs' halves of a slot landed
  uint64_t kv_empty[kT2Slots];  // each CTA: its half-slot may be refilled
  uint64_t s_full[2];           // each CTA: S_j of sub-tile x ready
  uint64_t p_full[2];           // leader: P_j of sub-tile x written in both CTAs
  uint64_t o_done[2];           // each CTA: last P.V of sub-tile x done
  uint64_t q_ready;             // leader: both CTAs' Q rows written
  uint32_t tmem_base;
  int abort;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kT2Threads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Tc2Bars bars;
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* q_s = smem;                     // [sub-tile][2 dim-halves][128 rows][128 B]
  uint8_t* slots = smem + 2 * kTcQBytes;   // [slot][16 KiB]

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const WorkItem it = a.items[blockIdx.x >> 1];
  const uint32_t* pages = a.pages + it.page_off;
  const int npages = it.npages;
  const int ntiles = (npages + kTcPagesPerTile - 1) / kTcPagesPerTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kT2Slots; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars.s_full[x], 1);
      mbar_init(&bars.p_full[x], 256);  // 128 rows in each CTA
      mbar_init(&bars.o_done[x], 1);
    }
    mbar_init(&bars.q_ready, 512);      // 256 Q rows in each CTA
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 64) prefetch_tmap(&kv_map);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote access
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;
  volatile int* abort = &bars.abort;

  if (warp == 0) {
    // -------------------------------------------------------------- producer
    const int64_t rows_total = (int64_t)a.num_pages * 2 * a.Hkv * kPageSize;
    const int pj = lane & (kTcPagesPerTile - 1);
    const bool mine = lane < kTcPagesPerTile;
    uint32_t cur = (mine && pj < npages) ? pages[pj] : 0xFFFFFFFFu;
    uint32_t nxt = 0xFFFFFFFFu;
    for (int idx = 0; idx < 2 * ntiles; ++idx) {
      const int s = idx % kT2Slots;
      const int j = idx >> 1, kv = idx & 1;
      if (kv == 0 && mine) {
        const int pn = (j + 1) * kTcPagesPerTile + pj;
        nxt = pn < npages ? pages[pn] : 0xFFFFFFFFu;
      }
      if (idx >= kT2Slots &&
          !mbar_wait_cl(&bars.kv_empty[s], ((idx / kT2Slots) - 1) & 1, abort, a.err))
        break;
      if (leader && lane == 0) mbar_arrive_expect_tx(&bars.kv_full[s], 2 * kT2SlotBytes);
      __syncwarp();
      const uint32_t bar = peer_addr(&bars.kv_full[s], 0);
      uint8_t* dst = slots + s * kT2SlotBytes;
      int y = (int)rows_total;  // absent page: past the end, TMA fills zeros
      if (mine && cur != 0xFFFFFFFFu) {
        if (cur < (uint32_t)a.num_pages)
          y = (int)((((int64_t)cur * 2 + kv) * a.Hkv + it.kv_head) * kPageSize);
        else
          report_error(a.err, kDevErrBadPage, cur);
      }
      if (kv == 0) {
        // K: this CTA's 4 pages, both dim-halves.
        if (mine && (pj >> 2) == (int)rank) {
          const int pl = pj & 3;
          tma_load_2d_pair(dst + pl * 2048, &kv_map, 0, y, bar);
          tma_load_2d_pair(dst + kT2KHalf + pl * 2048, &kv_map, 64, y, bar);
        }
      } else if (mine) {
        // V: this CTA's dim-half of all 8 pages.
        tma_load_2d_pair(dst + pj * 2048, &kv_map, 64 * (int)rank, y, bar);
      }
      if (kv == 1) cur = nxt;
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (leader && lane == 0 && ntiles > 0) {
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t slot_addr = smem_u32(slots);
      const uint64_t q_desc0 = umma_desc(q_addr, 16, 1024);
      const uint64_t k_desc0 = umma_desc(slot_addr, 16, 1024);
      const uint64_t v_desc0 = umma_desc(slot_addr, kT2SlotBytes, 1024);
      // The ring slot of idx is released only if some later idx reuses it.
      auto release = [&](int idx) {
        if (idx + kT2Slots < 2 * ntiles) umma2_commit_both(&bars.kv_empty[idx % kT2Slots]);
      };
      auto issue_qk = [&](int x, int j) {
        const uint64_t kd = k_desc0 + (uint64_t)((((2 * j) % kT2Slots) * kT2SlotBytes) >> 4);
        const uint64_t qd = q_desc0 + (uint64_t)((x * kTcQBytes) >> 4);
        const uint32_t d = tbase + col_s(x);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = (uint64_t)(((kk >> 2) * kT2KHalf + (kk & 3) * 32) >> 4);
          const uint64_t qoff = (uint64_t)(((kk >> 2) * (kTcQBytes / 2) + (kk & 3) * 32) >> 4);
          umma2_ss(d, qd + qoff, kd + off, kIdesc2QK, kk > 0 ? 1u : 0u);
        }
        umma2_commit_both(&bars.s_full[x]);
      };
      auto wait_slot = [&](int idx) {
        return mbar_wait_cl(&bars.kv_full[idx % kT2Slots], (idx / kT2Slots) & 1, abort, a.err);
      };
      bool ok = mbar_wait_cl(&bars.q_ready, 0, abort, a.err) && wait_slot(0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        issue_qk(1, 0);
        release(0);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const int sv = (2 * j + 1) % kT2Slots;
        const uint64_t vd = v_desc0 + (uint64_t)((sv * kT2SlotBytes) >> 4);
        for (int x = 0; ok && x < 2; ++x) {
          if (!mbar_wait_cl(&bars.p_full[x], j & 1, abort, a.err)) { ok = false; break; }
          if (x == 0 && !wait_slot(2 * j + 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tbase + col_o(x);
#pragma unroll
          for (int st = 0; st < 16; ++st) {
            const int kt = st & 7, part = st >> 3;  // hi terms, then lo terms
            const uint32_t pa = tbase + col_s(x) + (kt >> 2) * 64 + part * 32 + (kt & 3) * 8;
            umma2_ts(d, pa, vd + (uint64_t)((kt * 2048) >> 4), kIdesc2PV, (j > 0 || st > 0) ? 1u : 0u);
          }
          if (j + 1 < ntiles) {
            if (x == 0) {
              if (!wait_slot(2 * j + 2)) { ok = false; break; }
              tc_fence_after();
            }
            issue_qk(x, j + 1);
            if (x == 1) release(2 * j + 2);
          } else {
            umma2_commit_both(&bars.o_done[x]);
          }
        }
        if (ok) release(2 * j + 1);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int x = (warp - 2) >> 2;          // sub-tile: warps 2-5 -> A, 6-9 -> B
    const int quarter = warp & 3;           // TMEM lanes [32*quarter, +32)
    const int r = quarter * 32 + lane;      // row within the sub-tile
    const int row = (int)rank * 256 + x * 128 + r;  // row within the item
    const bool live = row < it.nrows;
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = lane_base + col_s(x);
    const uint32_t o_col = lane_base + col_o(x);
    const uint32_t q_ready_l = peer_addr(&bars.q_ready, 0);
    const uint32_t p_full_l = peer_addr(&bars.p_full[x], 0);
    {
      const uint4* src = nullptr;
      if (live) {
        const int rr = it.row0 + row, qi = rr / a.g;
        const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
        const int qid = a.qorder ? a.qorder[it.q_begin + qi] : it.q_begin + qi;
        src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.q) +
                                             ((size_t)qid * a.Hq + hq) * 128);
      }
      uint8_t* qx = q_s + x * kTcQBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = live ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qx + (c >> 3) * (kTcQBytes / 2) + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive_cluster(q_ready_l);
    }
    const float scale_log2 = a.scale_log2;
    float m_used = -INFINITY;
    uint64_t lsum = 0ull;
    for (int j = 0; j < ntiles; ++j) {
      bool ok = mbar_wait_cl(&bars.s_full[x], j & 1, abort, a.err);
      tc_fence_after();
      const int valid = (j == ntiles - 1) ? (npages - kTcPagesPerTile * j - 1) * kPageSize + it.last_valid
                                          : kTcTok;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float s[64];
        {
          float t[32];
          tmem_ld32(s_col + c * 64, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] = t[i];
          tmem_ld32(s_col + c * 64 + 32, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[32 + i] = t[i];
        }
        const int vc = valid - c * 64;
        if (vc < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= vc) s[i] = -INFINITY;
        }
        float m0 = s[0], m1 = s[1];
#pragma unroll
        for (int i = 2; i < 62; i += 4) {
          m0 = max3f(m0, s[i], s[i + 1]);
          m1 = max3f(m1, s[i + 2], s[i + 3]);
        }
        mx = max3f(mx, max3f(m0, m1, s[62]), s[63]);
      }
      float mt = mx * scale_log2;
      if (!ok) mt = m_used;
      if (__any_sync(0xffffffffu, mt > m_used + kRescaleThreshold)) {
        const float m_new = fmaxf(m_used, mt);
        const float f = fast_exp2(m_used - m_new);
        if (j > 0) {
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_scale32(o_col + c * 32, f);
        }
        lsum = f2_fma(lsum, f2_pack(f, f), 0ull);
        m_used = m_new;
      }
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_used, -m_used);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float s[64];
        {
          float t[32];
          tmem_ld32(s_col + c * 64, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] = t[i];
          tmem_ld32(s_col + c * 64 + 32, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[32 + i] = t[i];
        }
        const int vc = valid - c * 64;
        if (vc < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= vc) s[i] = -INFINITY;
        }
        softmax_chunk(s, sc2, nm2, lsum, s_col + c * 64);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_cluster(p_full_l);
    }
    {
      const float L = f2_lo(lsum) + f2_hi(lsum);
      int64_t slot = 0;
      if (live) {
        const int rr = it.row0 + row, qi = rr / a.g;
        const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
        slot = (int64_t)it.slot_base + (int64_t)qi * a.Hq + hq;
      }
      if (ntiles > 0) {
        mbar_wait_cl(&bars.o_done[x], 0, abort, a.err);
        tc_fence_after();
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (ntiles > 0) {
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (live) {
          float4* dst = reinterpret_cast<float4*>(a.part_o + slot * 128 + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        }
      }
      if (live) a.part_lse[slot] = L > 0.f ? m_used + log2f(L) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrival or product can still target this CTA
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols)
                 : "memory");
  }
}

int make_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int Hkv, int D,
                       int elem_bytes, int two_halves);

int launch_attn_tc2(const AttnArgs& a, int64_t num_pages, int num_items, cudaStream_t st) {
  if (a.D != 128 || a.kv_dtype != DD_DTYPE_BF16 || a.q_dtype != DD_DTYPE_BF16)
    return fail(DD_ERR_NOT_AVAILABLE, "CTA-pair tcgen05 path: bf16 KV and queries, head_dim 128");
  CUtensorMap map;
  int rc = make_kv_tensor_map(&map, a.kv, num_pages, a.Hkv, a.D, 2, 0);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(attn_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kT2Smem);
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_tc2 attribute: ") + cudaGetErrorString(e));
  {
    ProfScope ps(kProfTc, st);
    attn_tc2_kernel<<<2 * num_items, kT2Threads, kT2Smem, st>>>(map, a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_tc2 launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

}  // namespace dd
