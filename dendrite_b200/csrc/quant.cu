// KV-page quantisation to FP8 E4M3 (per K/V x KV-head scale) and MXFP8
// (E4M3 codes + one E8M0 exponent per 32 elements), and the round trip back.
//
// Reference semantics: QuantizedTensor::quantize computes
// scales = amax / 448 and data = clamp(t / scales, +-448) in f32 and keeps
// f32 data (crates/dendrite-core/src/quantization/fp8.rs:103-138); dequantize
// is data * scales (fp8.rs:141-152). Here the f32 quotient is rounded to a
// real E4M3 code (round to nearest even, saturating at 448 — the clamp), and
// candle's `tensor / f64` is an affine multiply by the reciprocal, so the
// default scale is amax * f32(1/448). MXFP8 (QuantFormat::MXFP8, block 32,
// crates/dendrite-core/src/quantization/mod.rs:57-59,133-140) has no reference
// code; it follows OCP MX v1.0: shared exponent floor(log2 amax) - emax(E4M3=8).
// All kernels are HBM-streaming: 16-byte vector loads, grid sized to the SMs.
#include "dd_device.cuh"

namespace dd {

__device__ __forceinline__ void load8(const void* src, int src_dtype, size_t i, float (&v)[8]) {
  if (src_dtype == DD_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + i);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + i);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = __uint_as_float(u[k] << 16);
      v[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
}

// Pass 1 of per-head E4M3: amax per (K/V, KV head) over the whole pool.
// One warp per page slice ([16][D] elements of one (page, K/V, head)); a
// lane's D/16 16-byte loads of a slice are issued together.
template <int D>
__global__ void amax_per_head_kernel(const void* src, int src_dtype, int64_t nslices, int Hkv,
                                     uint32_t* amax_bits) {
  __shared__ uint32_t sm[64];
  const int n2 = 2 * Hkv;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) sm[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr int per = kPageSize * D, kLoads = per / (32 * 8);
  for (int64_t s = warp0; s < nslices; s += nwarps) {
    float v[kLoads][8];
#pragma unroll
    for (int u = 0; u < kLoads; ++u) load8(src, src_dtype, (size_t)s * per + (u * 32 + lane) * 8, v[u]);
    float m = 0.f;
#pragma unroll
    for (int u = 0; u < kLoads; ++u)
#pragma unroll
      for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(v[u][k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) atomicMax(&sm[(uint32_t)s % (uint32_t)n2], __float_as_uint(m));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n2; i += blockDim.x)
    if (sm[i]) atomicMax(&amax_bits[i], sm[i]);
}

// Vectors (8 elements) per thread per round of the quantize kernels: their
// loads are issued before any is converted.
constexpr int kQuantUnroll = 4;

__device__ __forceinline__ float head_scale_from_amax(float amax, int mode) {
  if (!(amax > 0.f)) return 1.f;
  return mode == 0 ? amax * (float)(1.0 / 448.0) : __fdiv_rn(amax, 448.f);
}

// Pass 2: codes = E4M3_rn_sat(x / scale[kv][h]); block 0 also stores scales.
__global__ void quant_e4m3_kernel(const void* src, int src_dtype, int64_t nelem, int Hkv, int D,
                                  const uint32_t* amax_bits, int mode, uint8_t* codes,
                                  float* scales) {
  __shared__ float ssc[64];
  const int n2 = 2 * Hkv;
  for (int i = threadIdx.x; i < n2; i += blockDim.x)
    ssc[i] = head_scale_from_amax(__uint_as_float(amax_bits[i]), mode);
  __syncthreads();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < n2; i += blockDim.x) scales[i] = ssc[i];
  const int vec_shift = 31 - __clz(kPageSize * D / 8);  // vectors per page slice = 2 D
  const int64_t nvec = nelem / 8;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * kQuantUnroll;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x * kQuantUnroll; base < nvec; base += step) {
    float x[kQuantUnroll][8];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t v = base + u * blockDim.x + threadIdx.x;
      load8(src, src_dtype, (size_t)(v < nvec ? v : 0) * 8, x[u]);
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t v = base + u * blockDim.x + threadIdx.x;
      if (v >= nvec) continue;
      const size_t i = (size_t)v * 8;
      // Page slice of the vector (a slice is 2 D vectors, D a power of two).
      const float sc = ssc[(uint32_t)(v >> vec_shift) % (uint32_t)n2];
      float qv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) qv[k] = __fdiv_rn(x[u][k], sc);
      *reinterpret_cast<uint2*>(codes + i) =
          make_uint2(e4m3x4_satrn(qv[0], qv[1], qv[2], qv[3]), e4m3x4_satrn(qv[4], qv[5], qv[6], qv[7]));
    }
  }
}

// floor(log2(a)) of a finite a > 0 (normal or subnormal f32).
__device__ __forceinline__ int floor_log2_f32(float a) {
  const uint32_t b = __float_as_uint(a);
  const int e = (int)((b >> 23) & 0xff);
  if (e != 0) return e - 127;
  return (31 - __clz((int)(b & 0x7fffff))) - 149;
}

// MXFP8: 4 threads per 32-element block, each converting 8 elements.
__global__ void quant_mx_kernel(const void* src, int src_dtype, int64_t nelem, uint8_t* codes,
                                uint8_t* scales) {
  const int64_t nvec = nelem / 8;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * kQuantUnroll;
  // Warp-uniform trip count so the shuffles see the whole warp; the 4
  // threads of one 32-element block are always active together.
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x * kQuantUnroll; base < nvec; base += step) {
    float x[kQuantUnroll][8];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t v = base + u * blockDim.x + threadIdx.x;
      load8(src, src_dtype, (size_t)(v < nvec ? v : 0) * 8, x[u]);
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t v = base + u * blockDim.x + threadIdx.x;
      const size_t i = (size_t)(v < nvec ? v : 0) * 8;
      float m = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(x[u][k]));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      int e = m > 0.f ? floor_log2_f32(m) - 8 : -127;
      if (e < -127) e = -127;
      const float inv = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e, a normal f32
      const uint32_t lo = e4m3x4_satrn(x[u][0] * inv, x[u][1] * inv, x[u][2] * inv, x[u][3] * inv);
      const uint32_t hi = e4m3x4_satrn(x[u][4] * inv, x[u][5] * inv, x[u][6] * inv, x[u][7] * inv);
      if (v >= nvec) continue;
      *reinterpret_cast<uint2*>(codes + i) = make_uint2(lo, hi);
      if ((threadIdx.x & 3) == 0) scales[i / 32] = (uint8_t)(e + 127);
    }
  }
}

__global__ void dequant_kernel(const uint8_t* codes, int format, const void* scales, int64_t nelem,
                               int Hkv, int D, void* dst, int dst_dtype) {
  const int vec_shift = 31 - __clz(kPageSize * D / 8);  // vectors per page slice = 2 D
  const int64_t nvec = nelem / 8;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const size_t i = (size_t)v * 8;
    const uint2 c = *reinterpret_cast<const uint2*>(codes + i);
    float sc;
    if (format == DD_DTYPE_E4M3)
      sc = reinterpret_cast<const float*>(scales)[(uint32_t)(v >> vec_shift) % (uint32_t)(2 * Hkv)];
    else
      sc = e8m0_to_float(reinterpret_cast<const uint8_t*>(scales)[i / 32]);
    float y[8];
    const uint32_t w[2] = {c.x, c.y};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float2 a = e4m3x2_to_float2((uint16_t)(w[k] & 0xffff));
      const float2 b = e4m3x2_to_float2((uint16_t)(w[k] >> 16));
      y[4 * k] = a.x * sc; y[4 * k + 1] = a.y * sc;
      y[4 * k + 2] = b.x * sc; y[4 * k + 3] = b.y * sc;
    }
    if (dst_dtype == DD_DTYPE_F32) {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(dst) + i);
      o[0] = make_float4(y[0], y[1], y[2], y[3]);
      o[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + i) =
          make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                     pack_bf16x2(y[6], y[7]));
    }
  }
}

static int grid_for(int64_t work, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)sms * 8;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, cap));
}

static int check_qc(const dd_quant_config* qc) {
  if (!qc) return fail(DD_ERR_INVALID_ARGUMENT, "quant config is NULL");
  if (qc->format != DD_DTYPE_E4M3 && qc->format != DD_DTYPE_MXFP8)
    return fail(DD_ERR_INVALID_ARGUMENT, "format must be E4M3 or MXFP8");
  if (qc->src_dtype != DD_DTYPE_BF16 && qc->src_dtype != DD_DTYPE_F32)
    return fail(DD_ERR_INVALID_ARGUMENT, "src_dtype must be bf16 or f32");
  if (qc->head_dim != 64 && qc->head_dim != 128 && qc->head_dim != 256)
    return fail(DD_ERR_INVALID_ARGUMENT, "unsupported head_dim");
  if (qc->num_kv_heads <= 0 || qc->num_kv_heads > 32)
    return fail(DD_ERR_INVALID_ARGUMENT, "num_kv_heads must be in 1..32");
  if (qc->page_size != kPageSize) return fail(DD_ERR_INVALID_ARGUMENT, "page_size must be 16");
  if (qc->scale_mode != 0 && qc->scale_mode != 1)
    return fail(DD_ERR_INVALID_ARGUMENT, "scale_mode must be 0 or 1");
  return DD_OK;
}

}  // namespace dd

using namespace dd;

extern "C" size_t dd_quantize_workspace_size(const dd_quant_config* qc) {
  if (check_qc(qc)) return 0;
  return qc->format == DD_DTYPE_E4M3 ? kAlign : 0;
}

extern "C" int dd_quantize_kv_pages(const dd_quant_config* qc, const void* src, int64_t num_pages,
                                    uint8_t* codes, void* scales, void* workspace, size_t ws_bytes,
                                    dd_stream_t stream) {
  int rc = check_qc(qc);
  if (rc) return rc;
  if (num_pages < 0) return fail(DD_ERR_INVALID_ARGUMENT, "num_pages must be >= 0");
  if (num_pages == 0) return DD_OK;
  if (!src || !codes || !scales) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (((uintptr_t)src & 15) || ((uintptr_t)codes & 7))
    return fail(DD_ERR_INVALID_ARGUMENT, "src must be 16-byte and codes 8-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int Hkv = qc->num_kv_heads, D = qc->head_dim;
  const int64_t nelem = num_pages * 2 * Hkv * kPageSize * D;
  if (qc->format == DD_DTYPE_E4M3) {
    if (!workspace || ws_bytes < dd_quantize_workspace_size(qc))
      return fail(DD_ERR_WORKSPACE, "E4M3 quantization needs dd_quantize_workspace_size bytes");
    uint32_t* amax = reinterpret_cast<uint32_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(uint32_t) * 2 * Hkv, st);
    if (e != cudaSuccess) return fail(DD_ERR_CUDA, cudaGetErrorString(e));
    const int64_t nslices = num_pages * 2 * Hkv;
    { ProfScope ps(kProfQuant, st);
    const int ga = grid_for(nslices * 32, 256);
    if (D == 64) amax_per_head_kernel<64><<<ga, 256, 0, st>>>(src, qc->src_dtype, nslices, Hkv, amax);
    else if (D == 128) amax_per_head_kernel<128><<<ga, 256, 0, st>>>(src, qc->src_dtype, nslices, Hkv, amax);
    else amax_per_head_kernel<256><<<ga, 256, 0, st>>>(src, qc->src_dtype, nslices, Hkv, amax); }
    ProfScope ps(kProfQuant, st);
    quant_e4m3_kernel<<<grid_for(nelem / 8 / kQuantUnroll, 256), 256, 0, st>>>(
        src, qc->src_dtype, nelem, Hkv, D, amax, qc->scale_mode, codes,
        reinterpret_cast<float*>(scales));
  } else {
    ProfScope ps(kProfQuant, st);
    quant_mx_kernel<<<grid_for(nelem / 8 / kQuantUnroll, 256), 256, 0, st>>>(src, qc->src_dtype, nelem, codes,
                                                              reinterpret_cast<uint8_t*>(scales));
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, cudaGetErrorString(e));
  return DD_OK;
}

extern "C" int dd_dequantize_kv_pages(const dd_quant_config* qc, const uint8_t* codes,
                                      const void* scales, int64_t num_pages, void* dst,
                                      int32_t dst_dtype, dd_stream_t stream) {
  int rc = check_qc(qc);
  if (rc) return rc;
  if (dst_dtype != DD_DTYPE_BF16 && dst_dtype != DD_DTYPE_F32)
    return fail(DD_ERR_INVALID_ARGUMENT, "dst_dtype must be bf16 or f32");
  if (num_pages < 0) return fail(DD_ERR_INVALID_ARGUMENT, "num_pages must be >= 0");
  if (num_pages == 0) return DD_OK;
  if (!codes || !scales || !dst) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (((uintptr_t)dst & 15) || ((uintptr_t)codes & 7))
    return fail(DD_ERR_INVALID_ARGUMENT, "dst must be 16-byte and codes 8-byte aligned");
  const int64_t nelem = num_pages * 2 * qc->num_kv_heads * kPageSize * qc->head_dim;
  ProfScope ps(kProfQuant, (cudaStream_t)stream);
  dequant_kernel<<<grid_for(nelem / 8, 256), 256, 0, (cudaStream_t)stream>>>(
      codes, qc->format, scales, nelem, qc->num_kv_heads, qc->head_dim, dst, dst_dtype);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, cudaGetErrorString(e));
  return DD_OK;
}
