// CUDA-core partial attention over one work item: the path for f32 KV pages
// (TinyLlama-shaped parity config), head_dim 256, and f32 queries.
//
// Per page it stages K and V (dequantized to f32) in shared memory, computes
// the scaled scores of every row, does the online-softmax update and
// accumulates P.V — the arithmetic of ReferenceBackend::decode
// (crates/dendrite-core/src/attention/backend.rs:254-262: q.k^T * scale,
// softmax, .v) reorganised per page with a running max so that a node's pages
// are read once for all of its query rows. Output: the normalised partial
// output and its log2-domain LSE, merged later along each query's path.
#include "dd_device.cuh"

namespace dd {

constexpr int kSimpleRows = 64;
constexpr int kSimpleThreads = 256;

__device__ __forceinline__ float load_kv_elem(const AttnArgs& a, size_t idx, int kv, int h,
                                              uint32_t page, int t, int d) {
  switch (a.kv_dtype) {
    case DD_DTYPE_F32:
      return reinterpret_cast<const float*>(a.kv)[idx];
    case DD_DTYPE_BF16:
      return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(a.kv)[idx]);
    case DD_DTYPE_E4M3: {
      const float s = reinterpret_cast<const float*>(a.scales)[kv * a.Hkv + h];
      const float v = e4m3_to_float(reinterpret_cast<const uint8_t*>(a.kv)[idx]) * s;
      return __bfloat162float(__float2bfloat16_rn(v));
    }
    default: {  // MXFP8
      const size_t sidx = ((((size_t)page * 2 + kv) * a.Hkv + h) * kPageSize + t) * (a.D / 32) + d / 32;
      const float s = e8m0_to_float(reinterpret_cast<const uint8_t*>(a.scales)[sidx]);
      const float v = e4m3_to_float(reinterpret_cast<const uint8_t*>(a.kv)[idx]) * s;
      return __bfloat162float(__float2bfloat16_rn(v));
    }
  }
}

__global__ void __launch_bounds__(kSimpleThreads) attn_simple_kernel(AttnArgs a) {
  extern __shared__ float smem[];
  const int D = a.D;
  float* qs = smem;                       // [64][D]
  float* os = qs + kSimpleRows * D;       // [64][D]
  float* ks = os + kSimpleRows * D;       // [16][D]
  float* vs = ks + kPageSize * D;         // [16][D]
  float* sc = vs + kPageSize * D;         // [64][16]
  float* mrow = sc + kSimpleRows * kPageSize;
  float* lrow = mrow + kSimpleRows;
  float* arow = lrow + kSimpleRows;

  const uint32_t* pages;
  WorkItem it = resolve_item(a, pages, kSimpleRows);
  const bool causal = a.items && (it.nrows & kItemCausal) != 0;
  it.nrows &= kItemRowsMask;
  const int tid = threadIdx.x;
  const int nrows = it.nrows;
  if (nrows <= 0) return;

  // Stage the query rows.
  for (int idx = tid; idx < nrows * D; idx += kSimpleThreads) {
    const int r = idx / D, d = idx % D;
    const int rr = it.row0 + r, qi = rr / a.g;
    const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
    const int qid = a.qorder ? a.qorder[it.q_begin + qi] : it.q_begin + qi;
    const size_t qoff = ((size_t)qid * a.Hq + hq) * D + d;
    qs[idx] = a.q_dtype == DD_DTYPE_F32 ? reinterpret_cast<const float*>(a.q)[qoff]
                                        : bf16_bits_to_float(reinterpret_cast<const uint16_t*>(a.q)[qoff]);
    os[idx] = 0.f;
  }
  for (int r = tid; r < nrows; r += kSimpleThreads) {
    mrow[r] = -INFINITY;
    lrow[r] = 0.f;
  }
  __syncthreads();

  for (int pi = 0; pi < it.npages; ++pi) {
    const uint32_t page = pages[pi];
    int valid = (pi == it.npages - 1) ? it.last_valid : kPageSize;
    if (page >= (uint32_t)a.num_pages) {  // skip, as the reference skips unknown blocks
      if (tid == 0) report_error(a.err, kDevErrBadPage, page);
      valid = 0;
    }
    if (valid > 0) {
      for (int idx = tid; idx < kPageSize * D; idx += kSimpleThreads) {
        const int t = idx / D, d = idx % D;
        const size_t kidx = (((size_t)page * 2 + 0) * a.Hkv + it.kv_head) * kPageSize * D + idx;
        const size_t vidx = (((size_t)page * 2 + 1) * a.Hkv + it.kv_head) * kPageSize * D + idx;
        ks[idx] = load_kv_elem(a, kidx, 0, it.kv_head, page, t, d);
        vs[idx] = load_kv_elem(a, vidx, 1, it.kv_head, page, t, d);
      }
    }
    __syncthreads();
    if (valid == 0) continue;  // uniform across the block
    for (int idx = tid; idx < nrows * kPageSize; idx += kSimpleThreads) {
      const int r = idx / kPageSize, t = idx % kPageSize;
      float s = -INFINITY;
      const bool seen = !causal || pi * kPageSize + t < a.qlimit[it.q_begin + (it.row0 + r) / a.g];
      if (t < valid && seen) {
        float acc = 0.f;
        const float* qr = qs + r * D;
        const float* kr = ks + t * D;
        for (int d = 0; d < D; ++d) acc = fmaf(qr[d], kr[d], acc);
        s = acc * a.scale_log2;
      }
      sc[idx] = s;
    }
    __syncthreads();
    for (int r = tid; r < nrows; r += kSimpleThreads) {
      float mx = mrow[r];
      for (int t = 0; t < valid; ++t) mx = fmaxf(mx, sc[r * kPageSize + t]);
      const float alpha = exp2f(mrow[r] - mx);  // 0 when the old max is -inf
      float sum = 0.f;
      for (int t = 0; t < kPageSize; ++t) {
        const float p = t < valid ? exp2f(sc[r * kPageSize + t] - mx) : 0.f;
        sc[r * kPageSize + t] = p;
        sum += p;
      }
      lrow[r] = lrow[r] * alpha + sum;
      mrow[r] = mx;
      arow[r] = alpha;
    }
    __syncthreads();
    for (int idx = tid; idx < nrows * D; idx += kSimpleThreads) {
      const int r = idx / D, d = idx % D;
      float acc = os[idx] * arow[r];
      const float* pr = sc + r * kPageSize;
      for (int t = 0; t < valid; ++t) acc = fmaf(pr[t], vs[t * D + d], acc);
      os[idx] = acc;
    }
    __syncthreads();
  }

  // Normalised partial state per row.
  for (int idx = tid; idx < nrows * D; idx += kSimpleThreads) {
    const int r = idx / D, d = idx % D;
    const int rr = it.row0 + r, qi = rr / a.g;
    const int hq = qo_head_of(a.gqa_map, it.kv_head, rr % a.g, a.Hkv, a.g);
    const int64_t slot = (int64_t)it.slot_base + (int64_t)qi * a.Hq + hq;
    const float l = lrow[r];
    a.part_o[slot * D + d] = l > 0.f ? os[idx] / l : 0.f;
    if (d == 0) a.part_lse[slot] = l > 0.f ? mrow[r] + log2f(l) : -INFINITY;
  }
}

size_t simple_smem_bytes(int D) {
  return sizeof(float) * ((size_t)2 * kSimpleRows * D + 2 * kPageSize * D +
                          kSimpleRows * kPageSize + 3 * kSimpleRows);
}

cudaError_t launch_attn_simple(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  const size_t smem = simple_smem_bytes(a.D);
  cudaError_t e = cudaFuncSetAttribute(attn_simple_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  {
    ProfScope ps(kProfSimple, st);
    attn_simple_kernel<<<grid, kSimpleThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace dd
