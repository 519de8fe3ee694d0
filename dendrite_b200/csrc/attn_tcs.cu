// tcgen05 streaming attention for narrow cascade nodes (leaves and small
// shared nodes: <= 64 query rows), bf16 pages and queries, head_dim 128.
//
// The warp-level mma.sync kernel (attn_mma.cu) pays 48 legacy tensor-core
// instructions per page for a handful of query rows, which bounds it to
// ~50 GB/s per SM. Here the products run on the 5th-generation tensor core
// with the operands swapped so the many keys, not the few query rows, fill
// the M = 128 side:
//   S^T = K . Q^T     A = K tile (128 tokens x 128 dims, K-major, TMA),
//                     B = Q (N rows x 128 dims, K-major),  D = S^T in TMEM
//                     (lane = token, column = query row);
//   O^T += V^T . P^T  A = V tile read MN-major (dims on M), B = P^T in
//                     shared memory (tokens x N rows, MN-major), D = O^T
//                     (lane = dim, column = query row).
// Several work items of one KV head are packed into a group whose query
// rows share the N side (N <= 64) and whose pages stream back to back
// through one pipeline; a token's score counts only for the rows of its own
// item, so the cross-item products are masked to zero in the softmax.
//
// One persistent CTA per SM takes groups from a work counter:
//   warp 0      producer: 8 pages (two [16][64] boxes each) per K or V tile
//               into a 4-slot ring;
//   warp 1      TMEM (256 columns: S double buffer, O^T) and the products;
//   warps 2-5   one thread per token of a tile: scores of its item's rows,
//               lazy running max (per-row maxima are reduced only when some
//               score exceeds its row's max by 2^8), P as bf16 hi + lo terms
//               into the P^T buffer, per-thread partial row sums; at the end
//               of a group, one thread per dim writes the normalised rows.
// The arithmetic is ReferenceBackend::decode's
// (crates/dendrite-core/src/attention/backend.rs:254-262) over each item's
// tokens; the normalised partial state goes to the workspace for the merge.
//
// Status: parity-tested, but routed only in builds with DD_EXPERIMENT_TCS.
// Measured on B200 it streams ~4.6 TB/s on long leaves (31 GB/s per SM, the
// rate a 128 KiB TMA ring of 2 KiB boxes sustains per SM) against 6.4 TB/s
// for attn_mma.cu, so the default plan keeps the mma.sync kernel.
#include <algorithm>

#include "tc_common.cuh"

namespace dd {

constexpr int kSMaxRows = 32;
constexpr int kSMaxPages = 128;
constexpr int kSMaxItems = 32;
constexpr int kSSlots = 4;
constexpr int kSThreads = 192;
constexpr int kSPBuf = 128 * 128;          // P^T: 128 tokens x 128 B (rows padded to 64)
constexpr int kSQBytes = kSMaxRows * 256;  // Q: [2 dim-halves][32 rows][128 B]
constexpr int kSSmem = kSSlots * kTcSlotBytes + 4 * kSPBuf + kSQBytes + 1024;
constexpr uint32_t kSTmemCols = 256;
constexpr uint32_t kSColO = 128;

struct TcsShared {
  uint64_t kv_full[kSSlots];
  uint64_t kv_empty[kSSlots];
  uint64_t s_full[2];
  uint64_t o_done[2];
  uint64_t p_full;
  uint64_t q_ready;       // tables and Q of the group written (128 arrivals)
  uint64_t tables_ready;  // tables written (1 arrival; for the producer)
  uint32_t tmem_base;
  int abort;
  int32_t grp;            // group index, -1 when no work is left
  int32_t n_items, n_pages, n_rows, kv_head;
  uint32_t page_id[kSMaxPages];
  uint8_t page_item[kSMaxPages];
  uint8_t page_valid[kSMaxPages];
  int32_t item_row0[kSMaxItems + 1];  // rows of item i: [item_row0[i], item_row0[i+1])
  int32_t item_pos[kSMaxItems + 1];   // pages of item i in the group's page list
  int32_t item_poff[kSMaxItems];      // the item's first page in the plan's page list
  int32_t item_last[kSMaxItems];      // valid tokens of its last page
  int32_t item_rbase[kSMaxItems];     // its first row within the node (row0)
  int32_t item_qbeg[kSMaxItems];      // DFS position of the node's first query
  int32_t item_slot[kSMaxItems];      // partial-state slot base
  int32_t row_slot[kSMaxRows];
  const uint16_t* row_q[kSMaxRows];
  float m_used[kSMaxRows];
  float fac[kSMaxRows];
  float red[4][kSMaxRows];
};

// Barrier among `n` threads that also returns whether any of them passed
// `v` (the decision is the same in every thread).
__device__ __forceinline__ bool bar_any(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.cta.red.or.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Bounded wait that reports which wait site gave up (error aux = tag). With
// DD_EXPERIMENT_TIMING the cycles spent waiting are summed per site into the
// workspace header (u64 words 8-19 after pad[1]).
__device__ __forceinline__ bool wait_tag(uint64_t* bar, uint32_t parity, volatile int* abort,
                                         WsHeader* err, uint32_t tag) {
#ifdef DD_EXPERIMENT_TIMING
  const long long c0 = clock64();
  struct Acc {
    long long c0; WsHeader* e; uint32_t tg;
    __device__ ~Acc() {
      atomicAdd(reinterpret_cast<unsigned long long*>(&e->pad[1]) + 8 + ((tg >> 8) - 1) * 4 + (tg & 3),
                (unsigned long long)(clock64() - c0));
    }
  } acc{c0, err, tag};
#endif
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        report_error(err, kDevErrWaitTimeout, tag);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}

__global__ void __launch_bounds__(kSThreads, 1)
    attn_tcs_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a, const int32_t* groups,
                    int32_t num_groups) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ TcsShared sh;
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* slots = smem;                                  // [slot][2 dim-halves][128 tokens][128 B]
  uint8_t* pbuf = smem + kSSlots * kTcSlotBytes;          // [parity][hi, lo][128 tokens][128 B]
  uint8_t* q_s = pbuf + 4 * kSPBuf;                       // [2 dim-halves][64 rows][128 B]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSSlots; ++s) {
      mbar_init(&sh.kv_full[s], 1);
      mbar_init(&sh.kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.s_full[b], 1);
      mbar_init(&sh.o_done[b], 1);
    }
    mbar_init(&sh.p_full, 128);
    mbar_init(&sh.q_ready, 128);
    mbar_init(&sh.tables_ready, 1);
    sh.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sh.tmem_base)),
                 "r"(kSTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 64) prefetch_tmap(&kv_map);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sh.tmem_base;
  volatile int* abort = &sh.abort;
  uint32_t* claim = reinterpret_cast<uint32_t*>(&a.err->pad[0]);

  if (warp == 0) {
    // -------------------------------------------------------------- producer
    const int64_t rows_total = (int64_t)a.num_pages * 2 * a.Hkv * kPageSize;
    int sidx = 0;  // ring position, continuing across groups
    for (int gcount = 0;; ++gcount) {
      if (!wait_tag(&sh.tables_ready, gcount & 1, abort, a.err, 0x101)) break;
      if (sh.grp < 0) break;
      const int np = sh.n_pages, kvh = sh.kv_head;
      const int ntiles = (np + kTcPagesPerTile - 1) / kTcPagesPerTile;
      bool ok = true;
      for (int j = 0; ok && j < ntiles; ++j)
        for (int kv = 0; kv < 2; ++kv, ++sidx) {
          const int s = sidx % kSSlots;
          if (sidx >= kSSlots &&
              !wait_tag(&sh.kv_empty[s], ((sidx / kSSlots) - 1) & 1, abort, a.err, 0x102)) {
            ok = false;
            break;
          }
          if (lane == 0) mbar_arrive_expect_tx(&sh.kv_full[s], kTcSlotBytes);
          __syncwarp();
          if (lane < kTcPagesPerTile) {
            const int gp = j * kTcPagesPerTile + lane;
            int y = (int)rows_total;  // absent page: past the end, TMA fills zeros
            if (gp < np) {
              const uint32_t pid = sh.page_id[gp];
              if (pid < (uint32_t)a.num_pages)
                y = (int)((((int64_t)pid * 2 + kv) * a.Hkv + kvh) * kPageSize);
              else
                report_error(a.err, kDevErrBadPage, pid);
            }
            uint8_t* dst = slots + s * kTcSlotBytes + lane * 2048;
            tma_load_2d(dst, &kv_map, 0, y, &sh.kv_full[s]);
            tma_load_2d(dst + kTcHalfBytes, &kv_map, 64, y, &sh.kv_full[s]);
          }
        }
      if (!ok) break;
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t slot_addr = smem_u32(slots), p_addr = smem_u32(pbuf), q_addr = smem_u32(q_s);
      const uint64_t k_desc0 = umma_desc(slot_addr, 16, 1024);      // A: K, K-major
      const uint64_t v_desc0 = umma_desc(slot_addr, kTcHalfBytes, 1024);  // A: V^T, MN-major
      const uint64_t q_desc0 = umma_desc(q_addr, 16, 1024);         // B: Q, K-major
      const uint64_t p_desc0 = umma_desc(p_addr, 8192, 1024);       // B: P^T, MN-major
      int sidx = 0, gt = 0;
      for (int gcount = 0;; ++gcount) {
        if (!wait_tag(&sh.q_ready, gcount & 1, abort, a.err, 0x201)) break;
        if (sh.grp < 0) break;
        const int np = sh.n_pages;
        const int ntiles = (np + kTcPagesPerTile - 1) / kTcPagesPerTile;
        const uint32_t N = (uint32_t)max(16, (sh.n_rows + 15) & ~15);
        const uint32_t idesc_qk = (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((128u >> 4) << 24);
        const uint32_t idesc_pv = idesc_qk | (1u << 15) | (1u << 16);
        auto wait_slot = [&](int idx) {
          return wait_tag(&sh.kv_full[idx % kSSlots], (idx / kSSlots) & 1, abort, a.err, 0x202);
        };
        auto issue_qk = [&](int j) {
          const int ks = sidx + 2 * j;
          const uint64_t kd = k_desc0 + (uint64_t)(((ks % kSSlots) * kTcSlotBytes) >> 4);
          const uint32_t d = tbase + (uint32_t)((gt + j) & 1) * 64u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * kTcHalfBytes + (kk & 3) * 32) >> 4);
            const uint64_t qoff = (uint64_t)(((kk >> 2) * (kSQBytes / 2) + (kk & 3) * 32) >> 4);
            umma_ss(d, kd + off, q_desc0 + qoff, idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&sh.s_full[(gt + j) & 1]);
          umma_commit(&sh.kv_empty[ks % kSSlots]);
        };
        bool ok = true;
        for (int j = 0; ok && j < min(2, ntiles); ++j) {
          ok = wait_slot(sidx + 2 * j);
          tc_fence_after();
          if (ok) issue_qk(j);
        }
        for (int j = 0; ok && j < ntiles; ++j) {
          const int t = gt + j;
          if (!wait_tag(&sh.p_full, t & 1, abort, a.err, 0x203) || !wait_slot(sidx + 2 * j + 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int vs = (sidx + 2 * j + 1) % kSSlots;
          const uint64_t vd = v_desc0 + (uint64_t)((vs * kTcSlotBytes) >> 4);
          const uint64_t pd = p_desc0 + (uint64_t)(((t & 1) * 2 * kSPBuf) >> 4);
#pragma unroll
          for (int st = 0; st < 16; ++st) {
            const int kt = st & 7, part = st >> 3;  // hi terms, then lo terms
            umma_ss(tbase + kSColO, vd + (uint64_t)((kt * 2048) >> 4),
                    pd + (uint64_t)((part * kSPBuf + kt * 2048) >> 4), idesc_pv, (j > 0 || st > 0) ? 1u : 0u);
          }
          umma_commit(&sh.o_done[t & 1]);
          umma_commit(&sh.kv_empty[vs]);
          if (j + 2 < ntiles) {
            if (!wait_slot(sidx + 2 * (j + 2))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(j + 2);
          }
        }
        if (!ok) break;
        sidx += 2 * ntiles;
        gt += ntiles;
      }
    }
  } else {
    // ------------------------------------------------------- softmax / epilogue
    const int tid = threadIdx.x - 64;            // 0..127
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;           // token of a tile / dim of O^T (TMEM lane)
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const float scale_log2 = a.scale_log2;
    int gt = 0;
    for (int gcount = 0;; ++gcount) {
      // ---- claim a group and build its tables (page list, rows, Q)
      if (tid == 0) {
        const int32_t gi = (int32_t)atomicAdd(claim, 1u);
        sh.grp = gi < num_groups ? gi : -1;
        if (gi < num_groups) {
          sh.n_items = groups[4 * gi + 1];
          sh.n_pages = groups[4 * gi + 2];
          sh.n_rows = groups[4 * gi + 3];
          sh.kv_head = a.items[groups[4 * gi]].kv_head;
        }
      }
      named_bar_sync(1, 128);
      const int32_t gi = sh.grp;
      if (gi < 0) {
        if (tid == 0) mbar_arrive(&sh.tables_ready);
        mbar_arrive(&sh.q_ready);
        break;
      }
      const int n_items = sh.n_items, n_rows = sh.n_rows;
      const int first = groups[4 * gi];
      if (tid < n_items) {
        const WorkItem it = a.items[first + tid];
        sh.item_row0[tid + 1] = it.nrows;
        sh.item_pos[tid + 1] = it.npages;
        sh.item_poff[tid] = it.page_off;
        sh.item_last[tid] = it.last_valid;
        sh.item_rbase[tid] = it.row0;
        sh.item_qbeg[tid] = it.q_begin;
        sh.item_slot[tid] = it.slot_base;
      }
      named_bar_sync(1, 128);
      if (tid == 0) {
        sh.item_row0[0] = 0;
        sh.item_pos[0] = 0;
        for (int i = 0; i < n_items; ++i) {
          sh.item_row0[i + 1] += sh.item_row0[i];
          sh.item_pos[i + 1] += sh.item_pos[i];
        }
      }
      named_bar_sync(1, 128);
      // Page list and row table: one thread per page / row, so each needs a
      // single round trip to global memory.
      {
        const int np0 = sh.n_pages;
        for (int gp = tid; gp < np0; gp += 128) {
          int i = 0;
          while (i + 1 < n_items && sh.item_pos[i + 1] <= gp) ++i;
          const int k = gp - sh.item_pos[i];
          sh.page_id[gp] = a.pages[sh.item_poff[i] + k];
          sh.page_item[gp] = (uint8_t)i;
          sh.page_valid[gp] = (uint8_t)(gp == sh.item_pos[i + 1] - 1 ? sh.item_last[i] : kPageSize);
        }
        if (tid < n_rows) {
          int i = 0;
          while (i + 1 < n_items && sh.item_row0[i + 1] <= tid) ++i;
          const int rr = sh.item_rbase[i] + (tid - sh.item_row0[i]), qi = rr / a.g;
          const int hq = qo_head_of(a.gqa_map, sh.kv_head, rr % a.g, a.Hkv, a.g);
          const int qid = a.qorder ? a.qorder[sh.item_qbeg[i] + qi] : sh.item_qbeg[i] + qi;
          sh.row_slot[tid] = sh.item_slot[i] + qi * a.Hq + hq;
          sh.row_q[tid] = reinterpret_cast<const uint16_t*>(a.q) + ((size_t)qid * a.Hq + hq) * 128;
        }
      }
      if (tid < kSMaxRows) sh.m_used[tid] = -INFINITY;
      named_bar_sync(1, 128);
      if (tid == 0) mbar_arrive(&sh.tables_ready);
      // Q rows (zero beyond n_rows) into the K-major swizzled tile: 32 rows x 16
      // chunks of 16 B, 4 per thread.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = i * 128 + tid, r = ch >> 4, c = ch & 15;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < n_rows) v = reinterpret_cast<const uint4*>(sh.row_q[r])[c];
        *reinterpret_cast<uint4*>(q_s + (c >> 3) * (kSQBytes / 2) + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&sh.q_ready);

      const int np = sh.n_pages;
      const int ntiles = (np + kTcPagesPerTile - 1) / kTcPagesPerTile;
      const int N = max(16, (n_rows + 15) & ~15);
      float lsum[kSMaxRows];
#pragma unroll
      for (int r = 0; r < kSMaxRows; ++r) lsum[r] = 0.f;

      for (int j = 0; j < ntiles; ++j) {
        const int tt = gt + j;
        bool ok = wait_tag(&sh.s_full[tt & 1], (tt >> 1) & 1, abort, a.err, 0x301);
        tc_fence_after();
        // This thread's token: page p of the tile, its item and rows.
        const int gp = j * kTcPagesPerTile + (t >> 4);
        const bool live = gp < np && (t & 15) < sh.page_valid[min(gp, kSMaxPages - 1)];
        const int item = live ? sh.page_item[gp] : 0;
        const int ra = live ? sh.item_row0[item] : 0, rb = live ? sh.item_row0[item + 1] : 0;
        float x[kSMaxRows];
#pragma unroll
        for (int c = 0; c < kSMaxRows / 16; ++c) {
          if (c * 16 < N) {
            float v[16];
            tmem_ld16(lane_base + (uint32_t)(tt & 1) * 64u + c * 16, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) x[c * 16 + i] = v[i];
          }
        }
        tmem_wait_ld();
        bool over = false;
#pragma unroll
        for (int r = 0; r < kSMaxRows; ++r) {
          const bool mine = r >= ra && r < rb;
          x[r] = mine ? x[r] * scale_log2 : -INFINITY;
          over |= mine && x[r] > sh.m_used[r] + kRescaleThreshold;
        }
        if (!ok) over = false;
        if (bar_any(1, 128, over)) {
          // Row maxima of this tile, then the running max moves and O^T and
          // the partial sums are rescaled.
#pragma unroll
          for (int r = 0; r < kSMaxRows; ++r) {
            if (r < N) {
              float m = x[r];
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
              if (lane == 0) sh.red[quarter][r] = m;
            }
          }
          named_bar_sync(1, 128);
          if (tid < N) {
            const float tm = fmaxf(fmaxf(sh.red[0][tid], sh.red[1][tid]), fmaxf(sh.red[2][tid], sh.red[3][tid]));
            const float mo = sh.m_used[tid];
            const float mn = fmaxf(mo, tm);
            sh.fac[tid] = (mn == -INFINITY || mo == mn) ? 1.f : fast_exp2(mo - mn);
            sh.m_used[tid] = mn;
          }
          named_bar_sync(1, 128);
#pragma unroll
          for (int r = 0; r < kSMaxRows; ++r) lsum[r] *= sh.fac[r];
          if (j > 0) {
            // O^T holds P.V of tiles < j: wait for the last of them.
            wait_tag(&sh.o_done[(tt - 1) & 1], ((tt - 1) >> 1) & 1, abort, a.err, 0x302);
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < kSMaxRows / 16; ++c) {
              if (c * 16 < N) {
                float v[16];
                tmem_ld16(lane_base + kSColO + c * 16, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] *= sh.fac[c * 16 + i];
                tmem_st16(lane_base + kSColO + c * 16, v);
              }
            }
            tmem_wait_st();
          }
          named_bar_sync(1, 128);
        }
        // The P^T buffer of this parity was read by the products of tile tt-2.
        if (tt >= 2) wait_tag(&sh.o_done[tt & 1], ((tt - 2) >> 1) & 1, abort, a.err, 0x303);
        // P for this token: exp2(x - m) on its item's rows, 0 elsewhere,
        // written 8 rows (one 16-byte chunk of hi and of lo) at a time.
        uint8_t* prow = pbuf + (tt & 1) * 2 * kSPBuf + t * 128;
#pragma unroll
        for (int c = 0; c < kSMaxRows / 8; ++c) {  // the products read N <= 32 rows
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int r = 8 * c + 2 * k;
            float p0 = 0.f, p1 = 0.f;
            if (r >= ra && r < rb) p0 = fast_exp2(x[r] - sh.m_used[r]);
            if (r + 1 >= ra && r + 1 < rb) p1 = fast_exp2(x[r + 1] - sh.m_used[r + 1]);
            lsum[r] += p0;
            lsum[r + 1] += p1;
            split_bf16x2(p0, p1, hi[k], lo[k]);
          }
          const int sw = ((c ^ (t & 7)) << 4);
          *reinterpret_cast<uint4*>(prow + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(prow + kSPBuf + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&sh.p_full);
      }
      gt += ntiles;
      // ---- epilogue: row sums over the 128 threads, normalised O rows, LSE
#pragma unroll
      for (int r = 0; r < kSMaxRows; ++r) {
        if (r < N) {
          float s = lsum[r];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) sh.red[quarter][r] = s;
        }
      }
      if (ntiles > 0) {
        wait_tag(&sh.o_done[(gt - 1) & 1], ((gt - 1) >> 1) & 1, abort, a.err, 0x304);
        tc_fence_after();
      }
      named_bar_sync(1, 128);
      float o[kSMaxRows];
#pragma unroll
      for (int c = 0; c < kSMaxRows / 16; ++c) {
        if (c * 16 < N) {
          float v[16];
          if (ntiles > 0) {
            tmem_ld16(lane_base + kSColO + c * 16, v);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) o[c * 16 + i] = v[i];
        }
      }
      tmem_wait_ld();
#pragma unroll
      for (int r = 0; r < kSMaxRows; ++r) {
        if (r < n_rows) {
          const float L = sh.red[0][r] + sh.red[1][r] + sh.red[2][r] + sh.red[3][r];
          const int64_t slot = sh.row_slot[r];
          a.part_o[slot * 128 + t] = L > 0.f ? o[r] / L : 0.f;
          if (t == 0) a.part_lse[slot] = L > 0.f ? sh.m_used[r] + log2f(L) : -INFINITY;
        }
      }
      tc_fence_before();
      named_bar_sync(1, 128);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kSTmemCols)
                 : "memory");
  }
}

int make_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int Hkv, int D,
                       int elem_bytes, int two_halves);

int launch_attn_tcs(const AttnArgs& a, int64_t num_pages, const int32_t* groups, int num_groups,
                    int max_ctas, cudaStream_t st) {
  if (a.D != 128 || a.kv_dtype != DD_DTYPE_BF16 || a.q_dtype != DD_DTYPE_BF16)
    return fail(DD_ERR_NOT_AVAILABLE, "tcgen05 streaming path: bf16 KV and queries, head_dim 128");
  CUtensorMap map;
  int rc = make_kv_tensor_map(&map, a.kv, num_pages, a.Hkv, a.D, 2, 0);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(attn_tcs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmem);
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_tcs attribute: ") + cudaGetErrorString(e));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = std::max(1, std::min({num_groups, sms, max_ctas > 0 ? max_ctas : sms}));
  {
    ProfScope ps(kProfMma, st);
    attn_tcs_kernel<<<grid, kSThreads, kSSmem, st>>>(map, a, groups, num_groups);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_tcs launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

}  // namespace dd
