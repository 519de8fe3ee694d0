// tcgen05 (5th-generation tensor core, TMEM accumulators) partial attention
// for cascade nodes whose query rows form a dense contraction: the shared
// root and upper nodes of a tree, where hundreds to thousands of (query, GQA
// head) rows read the same pages.
//
// A work item is (node, KV head, 256-row tile, page range); each CTA runs the
// list the plan scheduled onto it (or one item, blockIdx.x), carrying the K/V
// ring, the barrier phases and its TMEM over from item to item. The rows
// form two 128-row sub-tiles A and B that share every K/V tile:
//   warp 0      TMA producer: K and V tiles of 128 tokens (8 pages x 2 boxes
//               of [16 tokens][64 dims], 128-byte swizzle) into the K/V
//               ring; lane p owns page p of each tile and reads its id one
//               tile ahead. FP8 pages go to a staging ring instead and warps
//               10-13 widen them to bf16 in the ring's layout.
//   warp 1      allocates all 512 TMEM columns; lane 0 issues every
//               tcgen05.mma and signals completion with tcgen05.commit, per
//               tile j in the order
//                 P_A.V_j, Q_A.K_{j+1}, P_B.V_j, Q_B.K_{j+1}
//               (S = Q.K^T: A = Q, B = K, both K-major smem; O += P.V: A = P
//               in TMEM, B = V MN-major), so the tensor core works on one
//               sub-tile while the softmax of the other runs (ping-pong).
//   warps 2-9   softmax, one thread per row: warps 2-5 own sub-tile A, 6-9
//               sub-tile B (a warp may only touch the TMEM lanes of its
//               quarter, warp % 4). One pass per 64-token chunk: its max,
//               exp2, row sum and P as two bf16 terms (hi + lo: P.V keeps
//               ~16 significant bits of P) written over the chunk's own
//               scores. The exponentials use a running integer reference
//               that moves only when a chunk's max passes it by more than 16
//               (log2 units); then O, the sum and the tile's earlier P are
//               scaled by the exact power of two, otherwise the stale
//               reference is kept, which is exact.
// TMEM columns: A: S/P 0-127, O 128-255; B: S/P 256-383, O 384-511. P_j
// overwrites S_j in place: S_{j+1} is committed after P.V_j, so when the
// softmax sees S_{j+1} the previous P has been consumed and O is final for
// a rescale. Each tcgen05.mma (M = N = 128, K = 16) occupies the tensor
// pipe ~90 cycles, so a 256-row tile keeps it busy for 48 of them per
// 128 tokens while each sub-tile's softmax has the other's 24 to run in.
//
// Causal (prefill) items mask each row's scores past its query's token
// limit in the softmax; their products still cover the item's tokens.
//
// The arithmetic is ReferenceBackend::decode's
// (crates/dendrite-core/src/attention/backend.rs:254-262) over the node's
// tokens; the normalised partial state goes to the workspace and is merged
// along each query's path by merge.cu.
#include "tc_common.cuh"

namespace dd {

constexpr int kTcRows = 256;            // rows per item: two sub-tiles of 128
constexpr int kTcStages = 3;                     // FP8 staging ring (K or V tile each)
constexpr int kTcStageCodes = kTcTok * 128;      // 128 tokens x 128 E4M3 codes
constexpr int kTcStageExps = kTcPagesPerTile * 64;  // MXFP8 exponents of a staged tile
// Staged codes keep the 128-byte swizzle of the TMA box, whose pattern
// follows shared-memory address bits 7-9: every stage starts on 1 KiB, and
// the exponents sit in their own area after the codes.
constexpr int kTcStageBytes = kTcStageCodes + kTcStageExps;

// Per KV dtype: bf16 pages are copied by TMA straight into the bf16 K/V ring;
// FP8 pages (E4M3 codes) are copied into a staging ring and two converter
// warps (10-13) widen them to bf16 in the ring's swizzled layout.
// FP8 converter warps (10-13). Four keep the widening ahead of the tensor
// pipe (two left the MXFP8 root ~25% slower); at 448 threads the kernel is
// held to 128 registers and spills ~90 bytes outside the inner loops.
constexpr int kTcConvWarps = 4;
template <int KV>
struct TcCfg {
  static constexpr bool kFp8 = KV != DD_DTYPE_BF16;
  static constexpr int kSlots = kFp8 ? 3 : 4;    // K/V ring slots (32 KiB each)
  static constexpr int kThreads = kFp8 ? 320 + 32 * kTcConvWarps : 320;
  static constexpr int kSmem =
      2 * kTcQBytes + kSlots * kTcSlotBytes + (kFp8 ? kTcStages * kTcStageBytes : 0) + 1024;
};
constexpr int kTcMaxSlots = 5;

struct TcBars {
  uint64_t kv_full[kTcMaxSlots];
  uint64_t kv_empty[kTcMaxSlots];
  uint64_t st_full[kTcStages];   // FP8 staging: codes landed
  uint64_t st_empty[kTcStages];  // FP8 staging: converted, reusable
  uint64_t s_full[2];            // per sub-tile: S_j ready (and P.V_{j-1} done)
  uint64_t p_full[2];            // per sub-tile: P_j written (128 arrivals)
  uint64_t item_done;            // every product of the current item complete
  uint64_t q_ready;              // both Q sub-tiles of the item in shared memory (256 arrivals)
  uint32_t tmem_base;
  int abort;
};

// Work item ii of this CTA's list (a.tc_order[ii] when the plan scheduled
// the items onto a fixed number of CTAs, else item ii itself).
__device__ __forceinline__ WorkItem tc_item(const AttnArgs& a, int ii) {
  return a.items[a.tc_order ? a.tc_order[ii] : ii];
}

template <int KV>
__global__ void __launch_bounds__(TcCfg<KV>::kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a) {
  constexpr int kTcSlots = TcCfg<KV>::kSlots;
  constexpr bool kFp8 = TcCfg<KV>::kFp8;
  extern __shared__ uint8_t smem_raw[];
  __shared__ TcBars bars;
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* q_s = smem;                       // [sub-tile][2 dim-halves][128 rows][128 B]
  uint8_t* slots = smem + 2 * kTcQBytes;     // [slot][2 dim-halves][128 rows][128 B]
  uint8_t* stages = slots + kTcSlots * kTcSlotBytes;  // FP8: [stage][128 rows][128 B]
  uint8_t* stage_exps = stages + kTcStages * kTcStageCodes;  // [stage][8 pages][64 B]

  // This CTA's items [ib, ie): a contiguous run of the plan's schedule, or
  // the single item blockIdx.x.
  const int ib = a.tc_cta_begin ? a.tc_cta_begin[blockIdx.x] : (int)blockIdx.x;
  const int ie = a.tc_cta_begin ? a.tc_cta_begin[blockIdx.x + 1] : (int)blockIdx.x + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A streaming kernel launched after this one as a programmatic dependent
  // may start once every CTA of this grid is running (it takes the other SMs).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcSlots; ++s) {
      mbar_init(&bars.kv_full[s], kFp8 ? 32 * kTcConvWarps : 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&bars.st_full[s], 1);
      mbar_init(&bars.st_empty[s], 32 * kTcConvWarps);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars.s_full[x], 1);
      mbar_init(&bars.p_full[x], 128);
    }
    mbar_init(&bars.item_done, 1);
    mbar_init(&bars.q_ready, 256);
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32 * 2) prefetch_tmap(&kv_map);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;
  volatile int* abort = &bars.abort;

  if (warp == 0) {
    // -------------------------------------------------------------- producer
    // Lane p < 8 owns page p of every tile and reads its id one tile ahead,
    // so no global read sits between the free-slot wait and the copies. The
    // ring runs on across items: gidx counts every K or V tile of the CTA.
    const int64_t rows_total = (int64_t)a.num_pages * 2 * a.Hkv * kPageSize;
    const int pj = lane & (kTcPagesPerTile - 1);
    const bool mine = lane < kTcPagesPerTile;
    int gidx = 0;
    bool ok = true;
    for (int ii = ib; ok && ii < ie; ++ii) {
      const WorkItem it = tc_item(a, ii);
      const uint32_t* pages = a.pages + it.page_off;
      const int npages = it.npages;
      const int ntiles = (npages + kTcPagesPerTile - 1) / kTcPagesPerTile;
      uint32_t cur = (mine && pj < npages) ? pages[pj] : 0xFFFFFFFFu;
      uint32_t nxt = 0xFFFFFFFFu;
      for (int idx = 0; idx < 2 * ntiles; ++idx, ++gidx) {
        const int j = idx >> 1, kv = idx & 1;
        if (kv == 0 && mine) {
          const int pn = (j + 1) * kTcPagesPerTile + pj;
          nxt = pn < npages ? pages[pn] : 0xFFFFFFFFu;
        }
        int y = (int)rows_total;  // absent page: past the end, TMA fills zeros
        bool ok_page = false;
        if (mine && cur != 0xFFFFFFFFu) {
          if (cur < (uint32_t)a.num_pages) {
            y = (int)((((int64_t)cur * 2 + kv) * a.Hkv + it.kv_head) * kPageSize);
            ok_page = true;
          } else {
            report_error(a.err, kDevErrBadPage, cur);
          }
        }
        if (kFp8) {
          // FP8: one box of [16 tokens][128 codes] per page into the staging
          // ring, plus the page's 64 MXFP8 exponent bytes.
          const int su = gidx % kTcStages;
          if (gidx >= kTcStages &&
              !mbar_wait(&bars.st_empty[su], ((gidx / kTcStages) - 1) & 1, abort, a.err)) {
            ok = false;
            break;
          }
          const int present = min(kTcPagesPerTile, npages - j * kTcPagesPerTile);
          if (lane == 0)
            mbar_arrive_expect_tx(&bars.st_full[su],
                                  kTcStageCodes + (KV == DD_DTYPE_MXFP8 ? 64 * present : 0));
          __syncwarp();
          if (mine) {
            tma_load_2d(stages + su * kTcStageCodes + pj * 2048, &kv_map, 0, y, &bars.st_full[su]);
            if (KV == DD_DTYPE_MXFP8 && pj < present) {
              // A bad page id still delivers its 64 bytes (from page 0) so the
              // transaction count completes; the error word marks the result.
              const int64_t ys = ok_page ? y : (int64_t)kv * a.Hkv * kPageSize;
              bulk_load(stage_exps + su * kTcStageExps + pj * 64,
                        reinterpret_cast<const uint8_t*>(a.scales) + ys * 4, 64, &bars.st_full[su]);
            }
          }
        } else {
          const int s = gidx % kTcSlots;
          if (gidx >= kTcSlots &&
              !mbar_wait(&bars.kv_empty[s], ((gidx / kTcSlots) - 1) & 1, abort, a.err)) {
            ok = false;
            break;
          }
          if (lane == 0) mbar_arrive_expect_tx(&bars.kv_full[s], kTcSlotBytes);
          __syncwarp();
          if (mine) {
            uint8_t* dst = slots + s * kTcSlotBytes;
            tma_load_2d(dst + pj * 2048, &kv_map, 0, y, &bars.kv_full[s]);
            tma_load_2d(dst + kTcHalfBytes + pj * 2048, &kv_map, 64, y, &bars.kv_full[s]);
          }
        }
        if (kv == 1) cur = nxt;
      }
      ok = __all_sync(0xffffffffu, ok);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    // Per tile j: P_A.V_j, Q_A.K_{j+1}, P_B.V_j, Q_B.K_{j+1}. Each P.V waits
    // for its sub-tile's softmax, which overlaps the other sub-tile's products.
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t slot_addr = smem_u32(slots);
      // Descriptors differ only in their start-address field (address >> 4).
      const uint64_t q_desc0 = umma_desc(q_addr, 16, 1024);
      const uint64_t k_desc0 = umma_desc(slot_addr, 16, 1024);
      const uint64_t v_desc0 = umma_desc(slot_addr, kTcHalfBytes, 1024);
      int g0 = 0;              // ring index of the item's first K tile
      int seen[2] = {0, 0};    // tiles each sub-tile's softmax has handed over
      bool ok = true;
      for (int ii = ib, n = 0; ok && ii < ie; ++ii, ++n) {
        WorkItem it = tc_item(a, ii);
        it.nrows &= kItemRowsMask;
        const int ntiles = (it.npages + kTcPagesPerTile - 1) / kTcPagesPerTile;
        const int nsub = it.nrows > 128 ? 2 : 1;
        auto issue_qk = [&](int x, int j) {
          const uint64_t kd = k_desc0 + (uint64_t)((((g0 + 2 * j) % kTcSlots) * kTcSlotBytes) >> 4);
          const uint64_t qd = q_desc0 + (uint64_t)((x * kTcQBytes) >> 4);
          const uint32_t d = tbase + col_s(x);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * kTcHalfBytes + (kk & 3) * 32) >> 4);
            const uint64_t qoff = (uint64_t)(((kk >> 2) * (kTcQBytes / 2) + (kk & 3) * 32) >> 4);
            umma_ss(d, qd + qoff, kd + off, kIdescQK, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars.s_full[x]);
        };
        auto wait_slot = [&](int idx) {
          return mbar_wait(&bars.kv_full[(g0 + idx) % kTcSlots], ((g0 + idx) / kTcSlots) & 1, abort,
                           a.err);
        };
        // Q of this item (written after the previous item's products completed).
        ok = mbar_wait(&bars.q_ready, n & 1, abort, a.err);
        if (!ok || ntiles == 0) continue;
        ok = wait_slot(0);
        if (!ok) break;
        tc_fence_after();
        for (int x = 0; x < nsub; ++x) issue_qk(x, 0);
        umma_commit(&bars.kv_empty[g0 % kTcSlots]);
        for (int j = 0; ok && j < ntiles; ++j) {
          const int sv = (g0 + 2 * j + 1) % kTcSlots;
          const uint64_t vd = v_desc0 + (uint64_t)((sv * kTcSlotBytes) >> 4);
          for (int x = 0; ok && x < nsub; ++x) {
            if (!(mbar_wait(&bars.p_full[x], (seen[x] + j) & 1, abort, a.err))) { ok = false; break; }
            if (x == 0 && !(wait_slot(2 * j + 1))) { ok = false; break; }
            tc_fence_after();
            const uint32_t d = tbase + col_o(x);
#pragma unroll
            for (int st = 0; st < 16; ++st) {
              const int kt = st & 7, part = st >> 3;  // hi terms, then lo terms
              const uint32_t pa = tbase + col_s(x) + (kt >> 2) * 64 + part * 32 + (kt & 3) * 8;
              umma_ts(d, pa, vd + (uint64_t)((kt * 2048) >> 4), kIdescPV, (j > 0 || st > 0) ? 1u : 0u);
            }
            if (j + 1 < ntiles) {
              if (x == 0) {
                if (!(wait_slot(2 * j + 2))) { ok = false; break; }
                tc_fence_after();
              }
              issue_qk(x, j + 1);
              if (x == nsub - 1) umma_commit(&bars.kv_empty[(g0 + 2 * j + 2) % kTcSlots]);
            }
          }
          if (ok) umma_commit(&bars.kv_empty[sv]);
        }
        // Every product of the item is complete when this arrives: O is final
        // and Q, S/P and O may be reused by the next item.
        if (ok) umma_commit(&bars.item_done);
        seen[0] += ntiles;
        if (nsub > 1) seen[1] += ntiles;
        g0 += 2 * ntiles;
      }
    }
  } else if (kFp8 && warp >= 10) {
    // ----------------------------------------------------------- converters
    // Thread t of 128 widens chunks id = t + 128 i (i < 8) of each staged tile:
    // chunk = 16 codes of one token (row), dims 16c..16c+15. Consecutive
    // threads cover two rows x four chunks of one dim-half, so each quarter
    // warp's two 16-byte stores hit eight distinct bank groups.
    const int t = threadIdx.x - 320;
    constexpr int kConvThreads = 32 * kTcConvWarps;
    int gidx = 0;
    bool ok = true;
    for (int ii = ib; ok && ii < ie; ++ii) {
      const WorkItem it = tc_item(a, ii);
      const int npages = it.npages;
      const int ntiles = (npages + kTcPagesPerTile - 1) / kTcPagesPerTile;
      for (int idx = 0; idx < 2 * ntiles; ++idx, ++gidx) {
        const int su = gidx % kTcStages, s = gidx % kTcSlots;
        if (!mbar_wait(&bars.st_full[su], (gidx / kTcStages) & 1, abort, a.err) ||
            (gidx >= kTcSlots &&
             !mbar_wait(&bars.kv_empty[s], ((gidx / kTcSlots) - 1) & 1, abort, a.err))) {
          ok = false;
          break;
        }
        const uint8_t* src = stages + su * kTcStageCodes;
        const uint8_t* exps = stage_exps + su * kTcStageExps;
        const float head_scale =
            KV == DD_DTYPE_E4M3 ? reinterpret_cast<const float*>(a.scales)[(idx & 1) * a.Hkv + it.kv_head] : 1.f;
        uint8_t* dst = slots + s * kTcSlotBytes;
        // Rows of absent pages hold zero codes but no exponents.
        const int live_rows = kPageSize * min(kTcPagesPerTile, npages - (idx >> 1) * kTcPagesPerTile);
#pragma unroll 4
        for (int id = t; id < 1024; id += kConvThreads) {
          const int cl = id & 3, half = (id >> 3) & 1;
          const int row = ((id >> 4) << 1) | ((id >> 2) & 1);
          const int c = half * 4 + cl;
          const uint4 codes = *reinterpret_cast<const uint4*>(src + row * 128 + ((c ^ (row & 7)) << 4));
          // Dequantised values are rounded to bf16 (the reference dequantises
          // pages to bf16 before attention).
          float mul = head_scale;
          if (KV == DD_DTYPE_MXFP8) mul = row < live_rows ? e8m0_to_float(exps[row * 4 + (c >> 1)]) : 1.f;
          uint32_t o[8];
          e4m3x16_to_bf16(codes, mul, o);
          uint8_t* drow = dst + half * kTcHalfBytes + row * 128;
          *reinterpret_cast<uint4*>(drow + (((2 * cl) ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(drow + (((2 * cl + 1) ^ (row & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars.kv_full[s]);
        mbar_arrive(&bars.st_empty[su]);
      }
    }
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------- softmax
    const int x = (warp - 2) >> 2;          // sub-tile: warps 2-5 -> A, 6-9 -> B
    const int quarter = warp & 3;           // TMEM lanes [32*quarter, +32)
    const int r = quarter * 32 + lane;      // row within the sub-tile
    const int row = x * 128 + r;            // row within the item
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = lane_base + col_s(x);
    const uint32_t o_col = lane_base + col_o(x);
    const float scale_log2 = a.scale_log2;
    int seen = 0;   // tiles of this sub-tile handed over so far (s_full / p_full phase)
    int done = 0;   // items with products so far (item_done phase)
    // Address of this thread's query row of item `iq` (NULL for a dead row).
    auto q_row = [&](const WorkItem& iq) -> const uint4* {
      if (row >= (iq.nrows & kItemRowsMask)) return nullptr;
      const int rr = iq.row0 + row, qi = rr / a.g;
      const int hq = qo_head_of(a.gqa_map, iq.kv_head, rr % a.g, a.Hkv, a.g);
      const int qid = a.qorder ? a.qorder[iq.q_begin + qi] : iq.q_begin + qi;
      return reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.q) +
                                            ((size_t)qid * a.Hq + hq) * 128);
    };
    // Q row -> the sub-tile's 128-byte-swizzled K-major tile, then hand the
    // tile to the MMA warp (the previous item's products are complete).
    auto write_q = [&](const WorkItem& iq) {
      const uint4* src = q_row(iq);
      uint8_t* qx = q_s + x * kTcQBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = src ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qx + (c >> 3) * (kTcQBytes / 2) + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars.q_ready);
    };
    if (ib < ie) write_q(tc_item(a, ib));
    for (int ii = ib; ii < ie; ++ii) {
      WorkItem it = tc_item(a, ii);
      const bool causal = (it.nrows & kItemCausal) != 0;
      it.nrows &= kItemRowsMask;
      const int npages = it.npages;
      const int ntiles = (npages + kTcPagesPerTile - 1) / kTcPagesPerTile;
      const bool live = row < it.nrows;
      const bool active = x == 0 || it.nrows > 128;
      if (ii + 1 < ie) {
        // The next item's query row into L2 while this item runs.
        const uint4* nq = q_row(tc_item(a, ii + 1));
        if (nq) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(nq));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(nq + 8));
        }
      }
      // Causal plans: tokens of the node this row sees (items start at the
      // node's first token).
      const int row_lim = causal && live ? a.qlimit[it.q_begin + (it.row0 + row) / a.g] : INT_MAX;
      float m_used = -INFINITY;
      uint64_t lsum = 0ull;  // running row sum, as two packed partial sums
      bool ok = true;
      for (int j = 0; active && j < ntiles; ++j) {
        ok = ok && mbar_wait(&bars.s_full[x], (seen + j) & 1, abort, a.err);
        tc_fence_after();
        const int valid = min((j == ntiles - 1) ? (npages - kTcPagesPerTile * j - 1) * kPageSize + it.last_valid
                                                : kTcTok,
                              row_lim == INT_MAX ? kTcTok : max(row_lim - kTcTok * j, 0));
        // One pass per 64-token chunk: the exponentials use the running
        // reference m_used (an integer, in log2 units), which moves only
        // when a chunk's max exceeds it by more than 16 (the first chunk of
        // the first tile always; later, practically never). Then O, the row
        // sum and the P this tile already holds are scaled by the exact power
        // of two 2^(m_used - m_new). P.V_{j-1} is complete here (S_j was
        // committed after it), so O can be rescaled in place; tcgen05.ld/st
        // are warp-wide, hence the warp-uniform decision (a factor of 1
        // leaves a row as is).
        const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
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
          // Raw scores times a positive scale: the max commutes.
          const float mt = ok ? max3f(m0, m1, fmaxf(s[62], s[63])) * scale_log2 : m_used;
          if (__any_sync(0xffffffffu, mt > m_used + kTcRescaleThreshold)) {
            const float m_new = mt > m_used + kTcRescaleThreshold ? ceilf(mt) : m_used;
            const float f = exp2f(m_used - m_new);  // a power of two; 0 when m_used is -inf
            if (j > 0) tmem_scale_cols<false>(o_col, 128, f);
            if (c == 1) tmem_scale_cols<true>(s_col, 64, f);  // chunk 0's P (hi, lo terms)
            lsum = f2_fma(lsum, f2_pack(f, f), 0ull);
            m_used = m_new;
          }
          softmax_chunk(s, sc2, f2_pack(-m_used, -m_used), lsum, s_col + c * 64);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars.p_full[x]);
      }
      if (active) seen += ntiles;
      // Every warp waits for the item's products before the next item's Q
      // overwrites its sub-tile (and, when active, to read O).
      if (ntiles > 0) {
        ok = mbar_wait(&bars.item_done, done & 1, abort, a.err) && ok;
        ++done;
        tc_fence_after();
      }
      // The next item's Q goes in before this epilogue, so its first
      // products overlap it (they write S; its first P.V, which overwrites
      // O, waits for this warp's P of that item, which comes after the
      // epilogue has read O).
      if (ii + 1 < ie && __all_sync(0xffffffffu, ok)) write_q(tc_item(a, ii + 1));
      // Epilogue: the normalised O row and its LSE.
      if (active) {
        const float L = f2_lo(lsum) + f2_hi(lsum);
        int64_t slot = 0;
        if (live) {
          const int rr = it.row0 + row, qi = rr / a.g;
          const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
          slot = (int64_t)it.slot_base + (int64_t)qi * a.Hq + hq;
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
      // O was read (tcgen05.wait::ld above) before this warp hands over the
      // next item's first P, after which P.V overwrites O.
      tc_fence_before();
      if (!__all_sync(0xffffffffu, ok)) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols)
                 : "memory");
  }
}

int make_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int Hkv, int D,
                       int elem_bytes, int two_halves);

int tc_row_tile() { return kTcRows; }

template <int KV>
static cudaError_t launch_tc_t(const CUtensorMap& map, const AttnArgs& a, int num_items,
                               cudaStream_t st) {
  constexpr int smem = TcCfg<KV>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<KV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem);
  if (e != cudaSuccess) return e;
  ProfScope ps(kProfTc, st);
  attn_tc_kernel<KV><<<num_items, TcCfg<KV>::kThreads, smem, st>>>(map, a);
  return cudaGetLastError();
}

int launch_attn_tc(const AttnArgs& a, int64_t num_pages, int grid, cudaStream_t st) {
  const bool fp8 = a.kv_dtype == DD_DTYPE_E4M3 || a.kv_dtype == DD_DTYPE_MXFP8;
  if (a.D != 128 || a.q_dtype != DD_DTYPE_BF16 || !(fp8 || a.kv_dtype == DD_DTYPE_BF16))
    return fail(DD_ERR_NOT_AVAILABLE, "tcgen05 path: bf16/E4M3/MXFP8 KV, bf16 queries, head_dim 128");
  if (a.kv_dtype == DD_DTYPE_MXFP8 && ((uintptr_t)a.scales & 15) != 0)
    return fail(DD_ERR_INVALID_ARGUMENT, "MXFP8 kv_scales must be 16-byte aligned");
  CUtensorMap map;
  int rc = make_kv_tensor_map(&map, a.kv, num_pages, a.Hkv, a.D, fp8 ? 1 : 2, 0);
  if (rc) return rc;
  cudaError_t e;
  switch (a.kv_dtype) {
    case DD_DTYPE_E4M3: e = launch_tc_t<DD_DTYPE_E4M3>(map, a, grid, st); break;
    case DD_DTYPE_MXFP8: e = launch_tc_t<DD_DTYPE_MXFP8>(map, a, grid, st); break;
    default: e = launch_tc_t<DD_DTYPE_BF16>(map, a, grid, st); break;
  }
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_tc launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

}  // namespace dd

extern "C" int dd_tc_available(void) { return 1; }
