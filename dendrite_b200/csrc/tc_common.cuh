// Shared pieces of the tcgen05 attention kernels (attn_tc.cu: one SM per
// 256-row tile; attn_tc2.cu: a CTA pair per 512-row tile): tile constants,
// UMMA shared-memory / instruction descriptors, TMEM load/store helpers and
// the per-chunk softmax that writes P over the scores.
#pragma once
#include "dd_device.cuh"

namespace dd {

constexpr int kTcTok = 128;             // tokens per tile
constexpr int kTcPagesPerTile = kTcTok / kPageSize;
constexpr int kTcSlotBytes = kTcTok * 128 * 2;   // 128 tokens x 128 dims bf16
constexpr int kTcHalfBytes = kTcTok * 128;       // one 64-dim half of a slot
constexpr int kTcQBytes = 128 * 128 * 2;         // one 128-row Q sub-tile
constexpr uint32_t kTmemCols = 512;
// Per sub-tile x: S (then P over it) at col_s(x), O at col_o(x).
__device__ __forceinline__ uint32_t col_s(int x) { return (uint32_t)x * 256u; }
__device__ __forceinline__ uint32_t col_o(int x) { return (uint32_t)x * 256u + 128u; }
constexpr float kRescaleThreshold = 8.0f;  // log2 units (attn_tc2.cu)
constexpr float kTcRescaleThreshold = 16.0f;  // log2 units (attn_tc.cu, single pass)

// Instruction descriptors, kind::f16, D f32, A/B bf16, M = 128, N = 128.
constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) |
                              ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 16);  // B (V) is MN-major

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread i gets columns [col, col+32) of lane i.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
      "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
      "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 32 columns of this thread's TMEM lane, times f, written back.
__device__ __forceinline__ void tmem_scale32(uint32_t taddr, float f) {
  float o[32];
  tmem_ld32(taddr, o);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint64_t v = f2_fma(f2_pack(o[i], o[i + 1]), f2_pack(f, f), 0ull);
    o[i] = f2_lo(v);
    o[i + 1] = f2_hi(v);
  }
  tmem_st32(taddr, o);
}

__device__ __forceinline__ void tmem_ld16u(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// `cols` columns (a multiple of 16) at taddr of this thread's lane, times f,
// 16 columns at a time: as f32 values, or (bf16x2) as two bf16 values each.
// With f a power of two the products are exact (within the formats' normal
// ranges). The rare rescale of the single-pass softmax; kept narrow so it
// needs few registers next to a live chunk of scores.
template <bool kBf16x2>
__device__ __noinline__ void tmem_scale_cols(uint32_t taddr, int cols, float f) {
  for (int c = 0; c < cols; c += 16) {
    uint32_t v[16];
    tmem_ld16u(taddr + c, v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      v[i] = kBf16x2 ? pack_bf16x2(__uint_as_float(v[i] << 16) * f, __uint_as_float(v[i] & 0xffff0000u) * f)
                     : __float_as_uint(__uint_as_float(v[i]) * f);
    tmem_st16u(taddr + c, v);
  }
  tmem_wait_st();
}

// Softmax of one 64-token chunk (s[], scores already masked): P = exp2(s *
// scale - m), accumulated into *acc, written as bf16 hi / lo terms into the
// chunk's own TMEM columns (hi: +0..31, lo: +32..63), which held its scores.
__device__ __forceinline__ void softmax_chunk(float (&s)[64], uint64_t sc2, uint64_t nm2,
                                              uint64_t& acc, uint32_t taddr) {
  uint64_t a0 = 0ull, a1 = 0ull;
#pragma unroll
  for (int i = 0; i < 64; i += 4) {
    const uint64_t x0 = f2_fma(f2_pack(s[i], s[i + 1]), sc2, nm2);
    const uint64_t x1 = f2_fma(f2_pack(s[i + 2], s[i + 3]), sc2, nm2);
    s[i] = fast_exp2(f2_lo(x0));
    s[i + 1] = fast_exp2(f2_hi(x0));
    s[i + 2] = fast_exp2(f2_lo(x1));
    s[i + 3] = fast_exp2(f2_hi(x1));
    a0 = f2_add(a0, f2_pack(s[i], s[i + 1]));
    a1 = f2_add(a1, f2_pack(s[i + 2], s[i + 3]));
  }
  acc = f2_add(acc, f2_add(a0, a1));
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      split_bf16x2_packed(f2_pack(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]), hi[i], lo[i]);
    tmem_st16u(taddr + c * 16, hi);
    tmem_st16u(taddr + 32 + c * 16, lo);
  }
}

}  // namespace dd
