// dd_decode_paged_static: paged batch decode that allocates nothing.
//
// Some callers cannot allocate device memory for the decode's scratch: a
// plugin that is handed only input/output pointers by a host engine that
// owns all device memory through its own pool, or a decode loop that must not
// call cudaMalloc (it synchronises the device and can fail under memory
// pressure). For them this entry point keeps its scratch (the split-K partial
// states and the device status words) in one file-scope __device__ array of
// kStaticScratchBytes, which every GPU that loads this library holds until
// the process exits. The kernels and their arithmetic are dd_decode_paged's;
// only where the scratch lives differs.
#include <mutex>

#include "dd_device.cuh"

namespace dd {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, looked up once per
// device. In host code the symbol's name is only a host-side stand-in, so the
// kernels are always given this address. The cached address outlives no
// device reset: after cudaDeviceReset the module is loaded again and the
// array may move (documented in the header).
static int static_scratch_ptr(void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DD_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(DD_ERR_NOT_AVAILABLE, "device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(DD_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return DD_OK;
}

}  // namespace dd

using namespace dd;

extern "C" int dd_decode_paged_static(const dd_attn_config* cfg, int32_t batch_size,
                                      int32_t max_pages_per_seq, const void* q,
                                      const void* kv_pages, const void* kv_scales,
                                      const int32_t* page_indptr, const int32_t* page_indices,
                                      const int32_t* num_tokens, void* out, float* lse,
                                      dd_stream_t stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (batch_size < 0 || max_pages_per_seq < 0)
    return fail(DD_ERR_INVALID_ARGUMENT, "bad batch size / max pages");
  const size_t need = dd_decode_paged_workspace_size(cfg, batch_size, max_pages_per_seq);
  if (need > kStaticScratchBytes)
    return fail(DD_ERR_WORKSPACE, "dd_decode_paged_static: this batch needs " + std::to_string(need) +
                                      " bytes of scratch but the static scratch holds " +
                                      std::to_string(kStaticScratchBytes) +
                                      " bytes; use dd_decode_paged with a caller workspace");
  void* scratch = nullptr;
  rc = static_scratch_ptr(&scratch);
  if (rc) return rc;
  // dd_decode_paged resets the status words at the head of the scratch and
  // overwrites every partial state it later reads, so no other clearing is
  // needed between calls.
  return dd_decode_paged(cfg, batch_size, max_pages_per_seq, q, kv_pages, kv_scales, page_indptr,
                         page_indices, num_tokens, out, lse, scratch, kStaticScratchBytes, stream);
}

extern "C" int dd_decode_paged_static_status(dd_stream_t stream, uint32_t* code, uint32_t* aux) {
  if (!code) return fail(DD_ERR_INVALID_ARGUMENT, "code is NULL");
  void* scratch = nullptr;
  const int rc = static_scratch_ptr(&scratch);
  if (rc) return rc;
  return dd_workspace_status(scratch, stream, code, aux);
}
