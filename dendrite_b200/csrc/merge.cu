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
  float m = -INFINITY, wsum = 0.f, acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int i = 0; i < n; ++i) {
    const int64_t slot = a.path_indptr ? (int64_t)a.path_slots[base + i] + h
                                       : ((int64_t)i * a.batch + p) * a.Hq + h;
    const float l = a.part_lse[slot];
    if (l == -INFINITY) continue;
    const float mn = fmaxf(m, l);
    const float sa = exp2f(m - mn), sb = exp2f(l - mn);
    const float* o = a.part_o + slot * D;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = acc[e] * sa + o[lane + 32 * e] * sb;
    wsum = wsum * sa + sb;
    m = mn;
  }
  const int q = a.qorder ? a.qorder[p] : p;
  const size_t ob = ((size_t)q * a.Hq + h) * D;
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float v = acc[e] * inv;
    if (a.out_dtype == DD_DTYPE_F32)
      reinterpret_cast<float*>(a.out)[ob + lane + 32 * e] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[ob + lane + 32 * e] = __float2bfloat16_rn(v);
  }
  if (a.lse && lane == 0)
    a.lse[(size_t)q * a.Hq + h] = wsum > 0.f ? (m + log2f(wsum)) * kLn2 : -INFINITY;
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
  // Outputs may alias inputs: each element reads its inputs before writing,
  // but lse is read by all D elements of a row, so go through a row-safe path
  // when l aliases la/lb: compute into o first, then write lse in a second pass.
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
