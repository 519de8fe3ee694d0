// Paged partial attention for cascade nodes with up to 16 query rows per
// work item (leaves, deep shared nodes, flat batch decode; wider nodes are
// cut into 16-row items), bf16 / E4M3 / MXFP8 KV.
//
// Persistent, multi-stream kernel. One CTA per SM holds kStreams independent
// streams, each with its own ring of shared-memory stages, one producer warp
// and one consumer warp (bf16) or two (FP8). Work items are claimed from a
// device counter (items are sorted longest first), one item at a time per
// stream.
//  - The stream's producer warp claims work, reads page ids a chunk ahead
//    (32 at a time, one per lane) and fills free stages with TMA
//    (cp.async.bulk.tensor), its lanes issuing a stage's copies in parallel:
//    one box per 16-token page slice of K or of V ([16][head_dim] contiguous
//    in the pool, 128-byte swizzle), plus a bulk copy of the item's query
//    rows into the stream's Q buffer. Pages read by one item only stream
//    L2 evict-first. Four streams per SM keep enough independent loads in
//    flight to run HBM near its random-read ceiling.
//  - FP8 pages land as 1-byte codes (+ E8M0 bytes for MXFP8) and stay FP8 in
//    shared memory: the consumers widen them (code * scale rounded to bf16)
//    straight into their mma fragments. Q.K^T contracts head dims in an order
//    where a lane's four K codes per k-step are one 4-byte word (Q is loaded
//    in the same order); for P.V a lane reads one word per token of four
//    tokens, transposes the 4x4 bytes and widens each head dim's four codes,
//    and the epilogue puts the head dims back in order. Widening makes a
//    consumer warp issue-bound, so FP8 streams have two: consumer h takes
//    page h of each stage, and consumer 1 hands its softmax state to
//    consumer 0 at the end of an item.
//  - A consumer owns all 16 query rows of its item (a GQA group of one or
//    more queries sharing the node). Per stage it takes two pages (32
//    tokens; one page each for an FP8 pair): q.k^T and p.v as m16n8k16 bf16
//    tensor-core tiles with f32 accumulators, online softmax in the log2
//    domain, P split into two bf16 terms so P.V keeps ~16 significant bits
//    of P. At the end of the item it writes one normalised partial state per
//    row straight from registers. Causal (prefill) items mask each row's
//    scores past its query's token limit.
// All waits are bounded mbarrier waits; a timeout sets an error word.
// The arithmetic is ReferenceBackend::decode's
// (crates/dendrite-core/src/attention/backend.rs:254-262) over the node's
// tokens; partial states are merged by merge.cu along each query's path.
#include <algorithm>

#include "dd_device.cuh"

namespace dd {

constexpr int kMmaRows = 16;       // query rows per work item
constexpr int kStepPages = 2;      // pages per stage
constexpr int kItemSlots = 2;      // item descriptors per stream

enum KvKind { kKvBf16 = 0, kKvE4m3 = 1, kKvMx = 2 };

template <int D, int KV>
struct MmaCfg {
  static constexpr int kSliceBf16 = kPageSize * D * 2;                 // one page, K or V
  static constexpr int kSliceRaw = KV == kKvBf16 ? kSliceBf16 : kPageSize * D;
  static constexpr int kMxBytes = KV == kKvMx ? kPageSize * (D / 32) : 0;
  // Stages are read in place by the consumer; FP8 stages are a quarter (E4M3)
  // of the bf16 ones, so the FP8 rings are deeper for the same bytes in flight.
  // bf16 streams have one consumer warp (consumer pairs for bf16, with 2
  // stages of 4 streams or 3 stages of 3 streams to fit shared memory,
  // measured slower: 142-146 us against 133 us on config 3).
  static constexpr bool kPair = KV != kKvBf16;
  static constexpr int kStreams = 4;  // independent streams per CTA
  static constexpr int kStages = KV == kKvBf16 ? 3 : 5;
  static constexpr int kRawStage = 2 * kStepPages * kSliceRaw;         // K0 K1 V0 V1
  static constexpr int kMxStage = 2 * kStepPages * kMxBytes;
  static constexpr int kStageAll = kRawStage;                          // 1 KiB multiple (swizzle)
  static constexpr int kExpBytes = kStages * kMxStage;                  // MXFP8 exponents, after the stages
  static constexpr int kQRowBytes = D * 2 + 16;                        // padded: conflict-free ldmatrix
  static constexpr int kQBytes = ((kMmaRows * kQRowBytes + 1023) / 1024) * 1024;
  static constexpr int kStreamBytes = ((kStages * kStageAll + kExpBytes + kQBytes + 1023) / 1024) * 1024;
  // FP8 streams have two consumer warps (the widening makes a consumer warp
  // issue-bound): consumer h takes page h of each stage, and at the end of an
  // item consumer 1 hands its softmax state to consumer 0 through kXBytes of
  // shared memory (68 floats per lane).
  static constexpr int kConsumers = kPair ? 2 * kStreams : kStreams;
  static constexpr int kThreads = (kConsumers + kStreams) * 32;  // consumers, then producers
  // Four consumer-pair streams: 384 threads, whose warpgroups (two of
  // consumers, one of producers) move registers to the consumers.
  static constexpr bool kSetMaxNreg = kPair && kStreams == 4;
  static constexpr int kXBytes = kPair ? (D / 2 + 4) * 32 * 4 : 0;
  static constexpr int kSmemBytes = kStreams * (kStreamBytes + kXBytes) + 1024;   // + alignment slack
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

// 3-D TMA load (x, y, z) into shared memory with mbarrier completion and an
// L2 eviction policy.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            int32_t z, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` (8 bf16 along D) of token row `t`
// inside a bf16 page slice stored as D/64 blocks of [16][128 B] with the
// 128-byte swizzle (chunk index XOR row % 8).
__device__ __forceinline__ uint32_t swz_bf16(int t, int chunk) {
  return (uint32_t)((chunk >> 3) * 2048 + t * 128 + (((chunk & 7) ^ (t & 7)) << 4));
}

// FP8 QK^T k order: k-step kk of lane c covers head dims fp8_kdim(kk, c) + 0..3
// (16-byte chunk c for k-steps 0-3, chunk c + 4 for 4-7), so the lane's four
// K codes of one token per k-step are one aligned 4-byte word.
__device__ __forceinline__ int fp8_kdim(int kk, int c) { return 16 * (c + 4 * (kk >> 2)) + 4 * (kk & 3); }

struct StageMeta {
  int8_t item_slot;
  int8_t flags;    // 1 first stage of an item, 2 last stage, 4 no more work
  int8_t np;       // pages in this stage (0..2)
  int8_t invalid;  // bit j: page j has an out-of-range id (skipped)
  int32_t page0;   // index of the stage's first page within the item
};
enum { kFirst = 1, kLast = 2, kDone = 4 };

constexpr int kMaxStages = 6;
struct StreamShared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t q_empty;
  uint64_t x_full, x_empty;  // FP8 consumer pairs: state handed over / read
  StageMeta meta[kMaxStages];
  WorkItem items[kItemSlots];
};

template <int D, int KV>
__global__ void __launch_bounds__(MmaCfg<D, KV>::kThreads, 1)
    attn_mma_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a) {
  using C = MmaCfg<D, KV>;
  static_assert(KV == kKvBf16 || D == 128, "FP8 fragments are laid out for head_dim 128");
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  constexpr int kStreams = C::kStreams;
  __shared__ StreamShared ss[kStreams];
  __shared__ int abort_flag;
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  constexpr int kCons = C::kConsumers;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < kStreams) {
    StreamShared& s = ss[threadIdx.x];
    for (int i = 0; i < S; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], C::kPair ? 2 : 1);
    }
    mbar_init(&s.q_empty, C::kPair ? 2 : 1);
    mbar_init(&s.x_full, 1);
    mbar_init(&s.x_empty, 1);
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x == kCons * 32) prefetch_tmap(&kv_map);
  __syncthreads();
  if (C::kSetMaxNreg) {
    // 384 threads launch at 168 registers (64,512); the producer warpgroup
    // gives up to 56 and the two consumer warpgroups take 224:
    // 128 x 56 + 256 x 224 = 64,512.
    if (warp >= kCons)
      asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
    else
      asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
  }

  if (warp >= kCons) {
    // ------------------------------------------------------------ producer
    // Producer warp kStreams + c drives stream c with all 32 lanes, so a
    // stall on one stream's reads never delays another stream. Lane l holds
    // the id of page chunk_base + l of the current item (and of the next
    // 32-page chunk), read 32 at a time one chunk ahead, so a stage issues no
    // dependent global read; lanes issue the stage's copies in parallel.
    const int c = warp - kCons;
    StreamShared& sh = ss[c];
    uint8_t* base = smem + c * C::kStreamBytes;
    uint8_t* qbuf = base + S * C::kStageAll + C::kExpBytes;
    int stage_idx = 0, item_count = 0;
    bool need_item = true, finished = false;
    WorkItem it{};
    const uint32_t* pages = nullptr;
    int pi = 0;                        // next page of the item
    int chunk_base = 0;                // first page of the chunk in cur_id
    uint32_t cur_id = 0, nxt_id = 0;   // lane l: ids of pages chunk_base + l, + 32
    int qid = 0;                       // lane r < nrows: query of the item's row r
    // The next item is prefetched one dependent read per stage (claim the
    // index, read the item, read its first 64 page ids and its rows' query
    // indices), and no step uses a value read in the same step, so the
    // latency chain overlaps the current item's stages.
    constexpr int kPfStates = 4;
    int pf_state = 0, pf_idx = 0;
    uint32_t pf_claim = 0;             // lane 0: claimed item index, in flight
    WorkItem pf_it{};
    bool pf_sole = false;              // the item is the only reader of its pages
    const uint32_t* pf_pages = nullptr;
    uint32_t pf_id = 0, pf_id2 = 0;
    int pf_qid = 0;                    // lane r < nrows: query index of row r
    auto pf_step = [&]() {
      if (pf_state == 0) {
        if (lane == 0) pf_claim = atomicAdd(&a.err->work_counter, 1u);
      } else if (pf_state == 1) {
        pf_idx = (int)__shfl_sync(0xffffffffu, pf_claim, 0);
        if (pf_idx < a.num_items) {
          pf_it = resolve_item_idx(a, pf_idx, pf_pages, kMmaRows);
          pf_sole = a.items ? (pf_it.nrows & kItemSoleReader) != 0 : a.row_tiles == 1;
          pf_it.nrows &= ~kItemSoleReader;  // the causal flag travels to the consumer
        }
      } else if (pf_state == 2) {
        if (pf_idx < a.num_items) {
          pf_id = lane < pf_it.npages ? pf_pages[lane] : 0u;
          pf_id2 = lane + 32 < pf_it.npages ? pf_pages[lane + 32] : 0u;
        }
      } else if (pf_state == 3) {
        if (pf_idx < a.num_items && lane < (pf_it.nrows & kItemRowsMask)) {
          const int qi = (pf_it.row0 + lane) / a.g;
          pf_qid = a.qorder ? a.qorder[pf_it.q_begin + qi] : pf_it.q_begin + qi;
        }
      }
      ++pf_state;
    };
    const uint64_t pol_first = l2_policy(true), pol_normal = l2_policy(false);
    uint64_t pol = pol_normal;
    uint64_t t_idle = global_ns();
    while (!finished) {
      if (abort_flag) break;
      bool done = false;
      if (need_item) {
        while (pf_state < kPfStates) pf_step();  // completes the prefetch (or all of it when disabled)
        done = pf_idx >= a.num_items;
        if (!done) {
          it = pf_it;
          pol = pf_sole ? pol_first : pol_normal;
          pages = pf_pages;
          pi = 0;
          chunk_base = 0;
          cur_id = pf_id;
          nxt_id = pf_id2;
          qid = pf_qid;
        }
        pf_state = 0;
      }
      // Wait (bounded, non-blocking poll) for a free stage.
      const int s = stage_idx % S;
      if (stage_idx >= S) {
        bool ok = true;
        while (!mbar_try_wait(&sh.empty[s], ((stage_idx / S) - 1) & 1)) {
          if (global_ns() - t_idle > kWaitLimitNs) {
            ok = false;
            break;
          }
        }
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) {
            abort_flag = 1;
            report_error(a.err, kDevErrWaitTimeout, 1);
          }
          break;
        }
      }
      // The Q buffer of the stream is reused once the consumer has read it.
      if (need_item && !done && item_count >= 1 &&
          !__all_sync(0xffffffffu, mbar_wait(&sh.q_empty, (item_count - 1) & 1, &abort_flag, a.err)))
        break;
      if (done) {
        if (lane == 0) {
          StageMeta m;
          m.item_slot = 0;
          m.flags = kDone;
          m.np = 0;
          m.invalid = 0;
          m.page0 = 0;
          sh.meta[s] = m;
          mbar_arrive_expect_tx(&sh.full[s], 0);
        }
        finished = true;
      } else {
        const int k = item_count & 1;
        const int np = min(kStepPages, it.npages - pi);
        // Ids of this stage's pages j < np from the lanes' chunk registers.
        uint32_t pg[kStepPages];
#pragma unroll
        for (int j = 0; j < kStepPages; ++j) {
          const int p = pi + j - chunk_base;  // 0..32
          const uint32_t x = __shfl_sync(0xffffffffu, cur_id, p & 31);
          const uint32_t y = __shfl_sync(0xffffffffu, nxt_id, p & 31);
          pg[j] = p < 32 ? x : y;
        }
        int invalid = 0;
#pragma unroll
        for (int j = 0; j < kStepPages; ++j)
          if (j < np && pg[j] >= (uint32_t)a.num_pages) {
            if (lane == 0) report_error(a.err, kDevErrBadPage, pg[j]);
            invalid |= 1 << j;
            pg[j] = 0;  // load something harmless; the consumer skips the page
          }
        const int nrows = it.nrows & kItemRowsMask;
        const uint32_t qbytes = need_item ? (uint32_t)nrows * D * 2 : 0u;
        const uint32_t bytes = (uint32_t)np * 2 * (C::kSliceRaw + C::kMxBytes) + qbytes;
        if (lane == 0) {
          if (need_item) sh.items[k] = it;
          StageMeta m;
          m.item_slot = (int8_t)k;
          m.flags = (int8_t)((need_item ? kFirst : 0) | (pi + np >= it.npages ? kLast : 0));
          m.np = (int8_t)np;
          m.invalid = (int8_t)invalid;
          m.page0 = pi;
          sh.meta[s] = m;
          mbar_arrive_expect_tx(&sh.full[s], bytes);
        }
        __syncwarp();
        // Lane r < nrows copies query row r; lane 16 + 2j + kv copies page
        // j's K (kv = 0) or V slice.
        if (qbytes && lane < nrows) {
          const int rr = it.row0 + lane;
          const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
          bulk_load(qbuf + lane * C::kQRowBytes,
                    reinterpret_cast<const uint16_t*>(a.q) + ((size_t)qid * a.Hq + hq) * D, D * 2,
                    &sh.full[s]);
        }
        const int l2 = lane - 16;
        if (l2 >= 0 && l2 < 2 * np) {
          const int j = l2 >> 1, kv = l2 & 1;
          const uint32_t pid = j == 0 ? pg[0] : pg[1];
          const int y = (int)((((int64_t)pid * 2 + kv) * a.Hkv + it.kv_head) * kPageSize);
          uint8_t* st = base + s * C::kStageAll;
          uint8_t* dst = st + (kv * kStepPages + j) * C::kSliceRaw;
          if (KV == kKvBf16 && D == 128)
            tma_load_3d(dst, &kv_map, 0, y, 0, &sh.full[s], pol);
          else
            tma_load_2d_hint(dst, &kv_map, 0, y, &sh.full[s], pol);
          if (KV == kKvMx)
            bulk_load_hint(base + S * C::kStageAll + s * C::kMxStage + (kv * kStepPages + j) * C::kMxBytes,
                           reinterpret_cast<const uint8_t*>(a.scales) + (size_t)y * (D / 32),
                           C::kMxBytes, &sh.full[s], pol);
        }
        pi += np;
        if (pi - chunk_base >= 32) {
          // Entering the next chunk: its ids are in nxt_id; read the one after.
          chunk_base += 32;
          cur_id = nxt_id;
          nxt_id = chunk_base + 32 + lane < it.npages ? pages[chunk_base + 32 + lane] : 0u;
        }
        if (need_item) need_item = false;
        if (pi >= it.npages) {
          need_item = true;
          ++item_count;
        }
      }
      ++stage_idx;
      t_idle = global_ns();
      if (!finished && pf_state < kPfStates) pf_step();
    }
  } else {
    // ------------------------------------------------------------ consumer
    const int cs = warp % kStreams, half = C::kPair ? warp / kStreams : 0;
    StreamShared& sh = ss[cs];
    uint8_t* base = smem + cs * C::kStreamBytes;
    float* xbuf = reinterpret_cast<float*>(smem + kStreams * C::kStreamBytes + cs * C::kXBytes);
    int pair_items = 0;  // items handed over (consumer 1) / taken over (consumer 0)
    uint8_t* qbuf = base + S * C::kStageAll + C::kExpBytes;
    WorkItem it{};
    uint32_t qa[D / 16][4];
    float o[D / 8][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float sc_k = 1.f, sc_v = 1.f;  // per-head E4M3 scales of the current item
    int lim0 = INT_MAX, lim1 = INT_MAX;  // causal plans: tokens seen by rows lane/4, +8
    const int tc = (lane & 3) * 2;

    for (int stage_idx = 0;; ++stage_idx) {
      const int s = stage_idx % S;
      if (!mbar_wait(&sh.full[s], (stage_idx / S) & 1, &abort_flag, a.err)) break;
      const StageMeta m = sh.meta[s];
      if (m.flags & kDone) break;
      if (m.flags & kFirst) {
        it = sh.items[m.item_slot];
        const bool causal = (it.nrows & kItemCausal) != 0;
        it.nrows &= kItemRowsMask;
        if (KV == kKvBf16) {
          const uint32_t qbase = smem_u32(qbuf);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int row = (lane & 7) + (((lane >> 3) & 1) << 3);
            const int chunk = kk * 2 + (lane >> 4);
            ldsm_x4(qbase + row * C::kQRowBytes + chunk * 16, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
          }
        } else {
          // FP8: k-step kk, k = 2c..2c+1 / 2c+8..2c+9 of lane c = lane % 4 is
          // head dim fp8_kdim(kk, c) + 0..1 / + 2..3, the order in which the
          // lane finds the codes of one token in one 4-byte word.
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int pd = fp8_kdim(kk, lane & 3);
            const uint2 r0 = *reinterpret_cast<const uint2*>(qbuf + (lane >> 2) * C::kQRowBytes + pd * 2);
            const uint2 r1 = *reinterpret_cast<const uint2*>(qbuf + ((lane >> 2) + 8) * C::kQRowBytes + pd * 2);
            qa[kk][0] = r0.x;
            qa[kk][1] = r1.x;
            qa[kk][2] = r0.y;
            qa[kk][3] = r1.y;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.q_empty);
#pragma unroll
        for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
        if (KV == kKvE4m3) {
          sc_k = reinterpret_cast<const float*>(a.scales)[it.kv_head];
          sc_v = reinterpret_cast<const float*>(a.scales)[a.Hkv + it.kv_head];
        }
        lim0 = lim1 = INT_MAX;
        if (causal) {
          const int r0 = lane >> 2, r1 = r0 + 8;
          lim0 = r0 < it.nrows ? a.qlimit[it.q_begin + (it.row0 + r0) / a.g] : INT_MAX;
          lim1 = r1 < it.nrows ? a.qlimit[it.q_begin + (it.row0 + r1) / a.g] : INT_MAX;
        }
      }
      const int np = m.np;
      const uint8_t* st = base + s * C::kStageAll;
      const uint8_t* kb;
      const uint8_t* vb;
      // A consumer pair splits the stage: consumer h takes page pj = h as
      // its page 0 (and no page 1).
      const int pj = C::kPair ? half : 0;
      kb = st + pj * C::kSliceRaw;
      vb = st + (kStepPages + pj) * C::kSliceRaw;
      // Valid tokens per page of the step (0 = absent or skipped).
      int valid[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        valid[j] = j < np ? ((m.page0 + j == it.npages - 1) ? it.last_valid : kPageSize) : 0;
        if ((m.invalid >> j) & 1) valid[j] = 0;
      }
      if (C::kPair) {
        valid[0] = valid[half];
        valid[1] = 0;
      }
      // MXFP8 exponent words of the stage, read before any code is widened:
      // kex[nt] = the four 32-dim blocks of K token nt*8 + lane/4, vex[j][i]
      // = those of V token 2c, 2c+1, 2c+8, 2c+9 (c = lane % 4) of page j.
      uint32_t kex[4] = {0u, 0u, 0u, 0u}, vex[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
      if (KV == kKvMx) {
        const uint8_t* mx = base + S * C::kStageAll + s * C::kMxStage;
#pragma unroll
        for (int nt = 0; nt < (C::kPair ? 2 : 4); ++nt)
          kex[nt] = *reinterpret_cast<const uint32_t*>(mx + (pj + (nt >> 1)) * C::kMxBytes +
                                                        ((nt & 1) * 8 + (lane >> 2)) * (D / 32));
#pragma unroll
        for (int j = 0; j < (C::kPair ? 1 : 2); ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            vex[j][i] = *reinterpret_cast<const uint32_t*>(
                mx + (kStepPages + pj + j) * C::kMxBytes + (2 * (lane & 3) + (i & 1) + 8 * (i >> 1)) * (D / 32));
      }
      if (valid[0] + valid[1] > 0) {
        // S = Q K^T for 16 rows x 32 tokens: four independent n-tile chains.
        float sacc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
        const bool two = valid[1] > 0;
        if (KV == kKvBf16) {
          const uint32_t k0 = smem_u32(kb), k1 = smem_u32(kb + C::kSliceBf16);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int t = ((lane >> 4) << 3) + (lane & 7);
            const int chunk = kk * 2 + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(k0 + swz_bf16(t, chunk), b0, b1, b2, b3);
            mma_bf16(sacc[0], qa[kk], b0, b1);
            mma_bf16(sacc[1], qa[kk], b2, b3);
            if (two) {
              ldsm_x4(k1 + swz_bf16(t, chunk), b0, b1, b2, b3);
              mma_bf16(sacc[2], qa[kk], b0, b1);
              mma_bf16(sacc[3], qa[kk], b2, b3);
            }
          }
        } else {
          // FP8 K straight from the stage: n-tile nt is tokens nt*8..+7; lane
          // (g, c) = (lane / 4, lane % 4) widens token nt*8 + g's codes of
          // 16-byte chunks c and c + 4 (k-steps 0-3 and 4-7) into the B
          // fragments. Odd tokens load chunk c + 4 first, so each 8-lane
          // phase of the 16-byte loads covers all 32 banks.
          const int c = lane & 3;
          uint4 kx[4], ky[4];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const int tp = (nt & 1) * 8 + (lane >> 2), odd = tp & 1;
            const uint8_t* row = kb + (nt >> 1) * C::kSliceRaw + tp * D;
            kx[nt] = *reinterpret_cast<const uint4*>(row + (((c + 4 * odd) ^ (tp & 7)) << 4));
            ky[nt] = *reinterpret_cast<const uint4*>(row + (((c + 4 - 4 * odd) ^ (tp & 7)) << 4));
          }
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            if (nt >= 2 && !two) break;
            const int odd = ((lane >> 2) & 1);
            const uint4 lo = odd ? ky[nt] : kx[nt], hi = odd ? kx[nt] : ky[nt];
            float mlo = sc_k, mhi = sc_k;
            if (KV == kKvMx) {
              mlo = e8m0_byte_to_float(kex[nt], c >> 1);
              mhi = e8m0_byte_to_float(kex[nt], 2 + (c >> 1));
            }
            const uint32_t wv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              uint32_t b0, b1;
              e4m3x4_to_bf16_cvt(wv[kk], kk < 4 ? mlo : mhi, b0, b1);
              mma_bf16(sacc[nt], qa[kk], b0, b1);
            }
          }
        }
        // x[nt][0..1]: row lane/4, tokens nt*8+tc+{0,1}; x[nt][2..3]: row +8.
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int vj = valid[nt >> 1];
          const int tok = (nt & 1) * 8 + tc;
          // Causal plans: token index within the node (items start at its
          // first token) against each row's limit.
          const int abs0 = (m.page0 + pj + (nt >> 1)) * kPageSize + tok;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const bool ok = tok + (c & 1) < vj && abs0 + (c & 1) < (c < 2 ? lim0 : lim1);
            sacc[nt][c] = ok ? sacc[nt][c] * a.scale_log2 : -INFINITY;
          }
          mx0 = fmaxf(mx0, fmaxf(sacc[nt][0], sacc[nt][1]));
          mx1 = fmaxf(mx1, fmaxf(sacc[nt][2], sacc[nt][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
        // Rescale the running state only when some row's max moved.
        if (__any_sync(0xffffffffu, nm0 != m0 || nm1 != m1)) {
          const float al0 = fast_exp2(m0 - nm0), al1 = fast_exp2(m1 - nm1);
          l0 *= al0;
          l1 *= al1;
#pragma unroll
          for (int n = 0; n < D / 8; ++n) {
            o[n][0] *= al0;
            o[n][1] *= al0;
            o[n][2] *= al1;
            o[n][3] *= al1;
          }
          m0 = nm0;
          m1 = nm1;
        }
        float p[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          p[nt][0] = fast_exp2(sacc[nt][0] - m0);
          p[nt][1] = fast_exp2(sacc[nt][1] - m0);
          p[nt][2] = fast_exp2(sacc[nt][2] - m1);
          p[nt][3] = fast_exp2(sacc[nt][3] - m1);
          l0 += p[nt][0] + p[nt][1];
          l1 += p[nt][2] + p[nt][3];
        }
        // O += P V, one 16-token k-step per page; P = P_hi + P_lo (bf16).
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (j == 1 && !two) break;
          uint32_t pa[4], pl[4];
          split_bf16x2(p[2 * j][0], p[2 * j][1], pa[0], pl[0]);
          split_bf16x2(p[2 * j][2], p[2 * j][3], pa[1], pl[1]);
          split_bf16x2(p[2 * j + 1][0], p[2 * j + 1][1], pa[2], pl[2]);
          split_bf16x2(p[2 * j + 1][2], p[2 * j + 1][3], pa[3], pl[3]);
          if (KV == kKvBf16) {
            const uint32_t vaddr = smem_u32(vb + j * C::kSliceBf16);
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
          } else {
            // FP8 V straight from the stage: lane (g, c) reads, per 32-dim
            // block b, dims 32b + 4g .. +3 of tokens 2c, 2c+1, 2c+8, 2c+9 (one
            // word each), transposes the 4x4 bytes, and widens dim d's four
            // codes into the B fragment of n-tile 4b + d, whose column g is
            // head dim 32b + 4g + d (fp8_odim).
            const uint8_t* vs = vb + j * C::kSliceRaw;
            const int g = lane >> 2, c = lane & 3;
            const int t0 = 2 * c, t1 = 2 * c + 1, t2 = 2 * c + 8, t3 = 2 * c + 9;
#pragma unroll
            for (int b = 0; b < D / 32; ++b) {
              const int off = 4 * (g & 3);
              const int ch = 2 * b + (g >> 2);
              const uint32_t w0 = *reinterpret_cast<const uint32_t*>(vs + t0 * D + ((ch ^ (t0 & 7)) << 4) + off);
              const uint32_t w1 = *reinterpret_cast<const uint32_t*>(vs + t1 * D + ((ch ^ (t1 & 7)) << 4) + off);
              const uint32_t w2 = *reinterpret_cast<const uint32_t*>(vs + t2 * D + ((ch ^ (t2 & 7)) << 4) + off);
              const uint32_t w3 = *reinterpret_cast<const uint32_t*>(vs + t3 * D + ((ch ^ (t3 & 7)) << 4) + off);
              const uint32_t a01 = __byte_perm(w0, w1, 0x5140), b01 = __byte_perm(w0, w1, 0x7362);
              const uint32_t a23 = __byte_perm(w2, w3, 0x5140), b23 = __byte_perm(w2, w3, 0x7362);
              const uint32_t u[4] = {__byte_perm(a01, a23, 0x5410), __byte_perm(a01, a23, 0x7632),
                                     __byte_perm(b01, b23, 0x5410), __byte_perm(b01, b23, 0x7632)};
              float m4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                m4[i] = KV == kKvMx ? e8m0_byte_to_float(vex[j][i], b) : sc_v;
#pragma unroll
              for (int d = 0; d < 4; ++d) {
                uint32_t b0, b1;
                e4m3x4_to_bf16_mul4(u[d], m4, b0, b1);
                mma_bf16(o[4 * b + d], pa, b0, b1);
                mma_bf16(o[4 * b + d], pl, b0, b1);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.empty[s]);
      if (m.flags & kLast) {
        if (C::kPair) {
          // Consumer 1 hands its (m, l, o) over; consumer 0 merges it into its
          // own (same fragment layout: lane-for-lane) and writes the state.
          if (half == 1) {
            if (pair_items > 0 && !mbar_wait(&sh.x_empty, (pair_items - 1) & 1, &abort_flag, a.err)) break;
#pragma unroll
            for (int n = 0; n < D / 8; ++n)
#pragma unroll
              for (int c = 0; c < 4; ++c) xbuf[(n * 4 + c) * 32 + lane] = o[n][c];
            xbuf[64 * 32 + lane] = m0;
            xbuf[65 * 32 + lane] = m1;
            xbuf[66 * 32 + lane] = l0;
            xbuf[67 * 32 + lane] = l1;
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.x_full);
            ++pair_items;
            continue;
          }
          if (!mbar_wait(&sh.x_full, pair_items & 1, &abort_flag, a.err)) break;
          const float pm0 = xbuf[64 * 32 + lane], pm1 = xbuf[65 * 32 + lane];
          const float M0 = fmaxf(m0, pm0), M1 = fmaxf(m1, pm1);
          const float fa0 = M0 == -INFINITY ? 0.f : fast_exp2(m0 - M0);
          const float fb0 = M0 == -INFINITY ? 0.f : fast_exp2(pm0 - M0);
          const float fa1 = M1 == -INFINITY ? 0.f : fast_exp2(m1 - M1);
          const float fb1 = M1 == -INFINITY ? 0.f : fast_exp2(pm1 - M1);
#pragma unroll
          for (int n = 0; n < D / 8; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              o[n][c] = o[n][c] * (c < 2 ? fa0 : fa1) + xbuf[(n * 4 + c) * 32 + lane] * (c < 2 ? fb0 : fb1);
          l0 = l0 * fa0 + xbuf[66 * 32 + lane] * fb0;
          l1 = l1 * fa1 + xbuf[67 * 32 + lane] * fb1;
          m0 = M0;
          m1 = M1;
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.x_empty);
          ++pair_items;
        }
        // Normalised partial state per row, written from registers.
        float L0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
        L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
        float L1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
        L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int r = (lane >> 2) + half * 8;
          if (r >= it.nrows) continue;
          const float L = half ? L1 : L0, M = half ? m1 : m0;
          const float inv = L > 0.f ? 1.f / L : 0.f;
          const int rr = it.row0 + r, qi = rr / a.g;
          const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
          const int64_t slot = (int64_t)it.slot_base + (int64_t)qi * a.Hq + hq;
          if (KV == kKvBf16) {
            float* dst = a.part_o + slot * D + tc;
#pragma unroll
            for (int n = 0; n < D / 8; ++n)
              *reinterpret_cast<float2*>(dst + n * 8) =
                  make_float2(o[n][2 * half] * inv, o[n][2 * half + 1] * inv);
          } else {
            // n-tile 4b + d, column 2c + e is head dim 32b + 8c + 4e + d.
            float* dst = a.part_o + slot * D + 8 * (lane & 3);
#pragma unroll
            for (int b = 0; b < D / 32; ++b)
#pragma unroll
              for (int e = 0; e < 2; ++e)
                *reinterpret_cast<float4*>(dst + 32 * b + 4 * e) =
                    make_float4(o[4 * b][2 * half + e] * inv, o[4 * b + 1][2 * half + e] * inv,
                                o[4 * b + 2][2 * half + e] * inv, o[4 * b + 3][2 * half + e] * inv);
          }
          if ((lane & 3) == 0) a.part_lse[slot] = L > 0.f ? M + log2f(L) : -INFINITY;
        }
      }
    }
  }
  // Launched as a programmatic dependent of the tcgen05 kernel (cascade
  // decode), this grid starts while that one runs, on the SMs it leaves free
  // and on each SM it gives up; it completes only after it, so the merge that
  // follows in the stream sees both kernels' partial states. Without a
  // prerequisite grid the wait returns at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
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

// View of the page pool as rows = num_pages * 2 * Hkv * 16 token rows of D
// elements with 128-byte swizzle. two_halves = 0: 2-D, box 16 rows x 128
// bytes. two_halves = 1 (bf16, D = 128): 3-D (64 dims, rows, 2 halves of a
// row) so one box of {64, 16, 2} moves a whole 4 KiB page slice, landing as
// [half][16 rows][128 B].
int make_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int Hkv, int D,
                       int elem_bytes, int two_halves) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(DD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const uint64_t rows = (uint64_t)num_pages * 2 * Hkv * kPageSize;
  if (rows == 0 || rows > 0x7FFFFFFFull)  // y coordinates are int32
    return fail(DD_ERR_INVALID_ARGUMENT, "page pool too large for a TMA descriptor");
  if (((uintptr_t)kv & 15) != 0) return fail(DD_ERR_INVALID_ARGUMENT, "kv_pages not 16-byte aligned");
  const CUtensorMapDataType dt =
      elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r;
  if (two_halves) {
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, 2};
    cuuint64_t strides[2] = {(cuuint64_t)D * elem_bytes, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)kPageSize, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    r = enc(map, dt, 3, const_cast<void*>(kv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)D * elem_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)kPageSize};
    cuuint32_t estr[2] = {1, 1};
    r = enc(map, dt, 2, const_cast<void*>(kv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(DD_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return DD_OK;
}

template <int D, int KV>
static cudaError_t launch_mma_t(const CUtensorMap& map, const AttnArgs& a, cudaStream_t st,
                               bool after_tc) {
  const int smem = MmaCfg<D, KV>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<D, KV>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if (MmaCfg<D, KV>::kSetMaxNreg) {
    // setmaxnreg.inc waits until the producers' setmaxnreg.dec has freed
    // enough registers: 128 x (R - 56) >= 256 x (224 - R) needs R >= 168 at
    // launch, so a build that allocates fewer must not launch.
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, attn_mma_kernel<D, KV>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs < 168) return cudaErrorInvalidConfiguration;
  }
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_mma_kernel<D, KV>, MmaCfg<D, KV>::kThreads, smem);
  if (e != cudaSuccess) return e;
  const int ctas_needed = (a.num_items + MmaCfg<D, KV>::kStreams - 1) / MmaCfg<D, KV>::kStreams;
  int grid = std::max(1, std::min(ctas_needed, sms * std::max(per_sm, 1)));
  ProfScope ps(kProfMma, st);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(MmaCfg<D, KV>::kThreads);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  if (after_tc) {
    // Programmatic dependent launch: the grid may start once every CTA of
    // the preceding tcgen05 kernel has started (it signals at its start).
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&lc, attn_mma_kernel<D, KV>, map, a);
}

bool mma_supported(int D, int kv_dtype) {
  if (kv_dtype == DD_DTYPE_BF16) return D == 64 || D == 128;
  if (kv_dtype == DD_DTYPE_E4M3 || kv_dtype == DD_DTYPE_MXFP8) return D == 128;
  return false;
}

int mma_row_tile() { return kMmaRows; }

// Launches the persistent kernel over a.num_items work items. The work
// counter in the workspace header must be zero (the caller resets the header).
int launch_attn_mma(const AttnArgs& a, int64_t num_pages, cudaStream_t st, bool after_tc) {
  if (a.num_items <= 0) return DD_OK;
  CUtensorMap map;
  const int eb = a.kv_dtype == DD_DTYPE_BF16 ? 2 : 1;
  int rc = make_kv_tensor_map(&map, a.kv, num_pages, a.Hkv, a.D, eb,
                              a.kv_dtype == DD_DTYPE_BF16 && a.D == 128);
  if (rc) return rc;
  cudaError_t e;
  if (a.kv_dtype == DD_DTYPE_BF16)
    e = a.D == 64 ? launch_mma_t<64, kKvBf16>(map, a, st, after_tc) : launch_mma_t<128, kKvBf16>(map, a, st, after_tc);
  else if (a.kv_dtype == DD_DTYPE_E4M3)
    e = launch_mma_t<128, kKvE4m3>(map, a, st, after_tc);
  else
    e = launch_mma_t<128, kKvMx>(map, a, st, after_tc);
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("attn_mma launch: ") + cudaGetErrorString(e));
  return DD_OK;
}

}  // namespace dd
