// Log-sum-exp merge of partial attention states.
//
// merge_attention_outputs (crates/dendrite-ffi/src/flashinfer/cascade.rs:116-124)
// combines two states: m = max(l1, l2), o = (o1 e^{l1-m} + o2 e^{l2-m}) /
// (e^{l1-m} + e^{l2-m}), lse = m + ln(sum). Here the same combination runs over
// every partial state on a query's root-to-leaf path (all chunks of all
// cascade nodes), one warp per (query, head), with each lane owning D/32
// elements; partial LSEs are kept in the log2 domain internally and the
// output LSE is natural-log like the reference's.
#include "dd_device.cuh"

namespace dd {


// One warp per (query, head). Lanes first fetch the slot ids and LSEs of up
// to 32 path entries at once and reduce max / weights with shuffles; the
// outputs are then accumulated with independent vector loads (lane owns E
// consecutive elements), so no load waits on another.
template <int D>
__global__ void __launch_bounds__(256) merge_paths_kernel(MergeArgs a) {
  constexpr int E = D / 32;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.batch * a.Hq) return;
  const int p = warp / a.Hq, h = warp % a.Hq;
  int n;
  int32_t base = 0;
  if (a.path_indptr) {
    base = a.path_indptr[p];
    n = a.path_indptr[p + 1] - base;
  } else {
    n = a.nsplit;
  }
  float M = -INFINITY, W = 0.f, acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int c0 = 0; c0 < n; c0 += 32) {
    const int i = c0 + lane;
    int64_t slot = 0;
    float l = -INFINITY;
    if (i < n) {
      slot = a.path_indptr ? (int64_t)a.path_slots[base + i] + h : ((int64_t)i * a.batch + p) * a.Hq + h;
      l = a.part_lse[slot];
    }
    float cm = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    if (cm == -INFINITY) continue;  // nothing in this chunk
    const float nm = fmaxf(M, cm);
    const float f = exp2f(M - nm);  // 0 when M is -inf
    M = nm;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] *= f;
    float w = l == -INFINITY ? 0.f : exp2f(l - M);
    float ws = w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
    W = W * f + ws;
    const int cn = min(32, n - c0);
#pragma unroll 4
    for (int k = 0; k < cn; ++k) {
      const float wk = __shfl_sync(0xffffffffu, w, k);
      const int64_t sk = __shfl_sync(0xffffffffu, slot, k);
      if (wk == 0.f) continue;
      const float* o = a.part_o + sk * D + lane * E;
      if (E == 4) {
        const float4 v = *reinterpret_cast<const float4*>(o);
        acc[0] += wk * v.x; acc[1] += wk * v.y; acc[2] += wk * v.z; acc[3] += wk * v.w;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += wk * o[e];
      }
    }
  }
  const int q = a.qorder ? a.qorder[p] : p;
  const size_t ob = ((size_t)q * a.Hq + h) * D + lane * E;
  const float inv = W > 0.f ? 1.f / W : 0.f;
  if (a.peer_out) {
    // Head split: the row goes to its global head in every rank's output
    // (NVLink stores into peer memory; local head h of rank r under the
    // GQA map restricted to the rank's KV heads).
    const int Hkv_r = a.Hkv_global / a.world, k0 = a.rank * Hkv_r, g = a.Hq_global / a.Hkv_global;
    const int hg = a.gqa_map == DD_GQA_TILED ? (k0 + h % Hkv_r) + (h / Hkv_r) * a.Hkv_global : k0 * g + h;
    const size_t og = ((size_t)q * a.Hq_global + hg) * D + lane * E;
    for (int r = 0; r < a.world; ++r) {
      if (a.out_dtype == DD_DTYPE_F32) {
#pragma unroll
        for (int e = 0; e < E; ++e) reinterpret_cast<float*>(a.peer_out[r])[og + e] = acc[e] * inv;
      } else {
#pragma unroll
        for (int e = 0; e < E; e += 2)
          *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(a.peer_out[r]) + og + e) =
              pack_bf16x2(acc[e] * inv, acc[e + 1] * inv);
      }
    }
  } else if (a.out_dtype == DD_DTYPE_F32) {
#pragma unroll
    for (int e = 0; e < E; ++e) reinterpret_cast<float*>(a.out)[ob + e] = acc[e] * inv;
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(a.out) + ob + e) =
          pack_bf16x2(acc[e] * inv, acc[e + 1] * inv);
  }
  if (a.lse && lane == 0)
    a.lse[(size_t)q * a.Hq + h] = W > 0.f ? (M + log2f(W)) * kLn2 : -INFINITY;
}

cudaError_t launch_merge(const MergeArgs& a, cudaStream_t st) {
  const int64_t warps = (int64_t)a.batch * a.Hq;
  if (warps == 0) return cudaSuccess;
  const int blocks = (int)((warps * 32 + 255) / 256);
  ProfScope ps(kProfMerge, st);
  switch (a.D) {
    case 64: merge_paths_kernel<64><<<blocks, 256, 0, st>>>(a); break;
    case 128: merge_paths_kernel<128><<<blocks, 256, 0, st>>>(a); break;
    default: merge_paths_kernel<256><<<blocks, 256, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

// Element-wise two-state merge in the natural-log convention of
// merge_attention_outputs, over n rows of D.
__global__ void merge_two_kernel(int32_t n, int32_t D, const float* oa, const float* la,
                                 const float* ob, const float* lb, float* o, float* l) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * D) return;
  const int64_t r = i / D;
  const float l1 = la[r], l2 = lb[r];
  const float mx = fmaxf(l1, l2);
  float e1 = expf(l1 - mx), e2 = expf(l2 - mx);
  if (mx == -INFINITY) e1 = e2 = 0.f;
  const float s = e1 + e2;
  const float v = s > 0.f ? (oa[i] * e1 + ob[i] * e2) / s : 0.f;
  o[i] = v;
  if (i % D == 0) l[r] = s > 0.f ? mx + logf(s) : -INFINITY;
}

}  // namespace dd

extern "C" int dd_merge_states(int32_t n, int32_t D, const float* oa, const float* la,
                               const float* ob, const float* lb, float* o, float* l,
                               dd_stream_t stream) {
  using namespace dd;
  if (n < 0 || D <= 0) return fail(DD_ERR_INVALID_ARGUMENT, "bad sizes");
  if (n == 0) return DD_OK;
  if (!oa || !la || !ob || !lb || !o || !l) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  // o may alias oa or ob (each element reads its inputs before writing it),
  // but every element of a row reads la/lb, so l may not alias them.
  const int64_t total = (int64_t)n * D;
  const int threads = 256;
  const int blocks = (int)((total + threads - 1) / threads);
  if (l == la || l == lb) {
    return fail(DD_ERR_INVALID_ARGUMENT, "lse output may not alias an lse input");
  }
  {
    ProfScope ps(kProfMerge, (cudaStream_t)stream);
    merge_two_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(n, D, oa, la, ob, lb, o, l);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, cudaGetErrorString(e));
  return DD_OK;
}
