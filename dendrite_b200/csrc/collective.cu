// The collective of the KV-head split (one long tree over W GPUs): an NCCL
// all-gather of every rank's [batch][Hq/W][D] output over NVLink, then the
// head reorder of dd_scatter_head_shards.
//
// The library does not link NCCL: a caller (the Rust engine, or a Python
// process whose torch already loaded NCCL) owns the communicator, and
// ncclAllGather is looked up at run time in the NCCL library already loaded
// into the process (the one that created the communicator), falling back to
// loading libnccl.so.2.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "dd_device.cuh"

namespace dd {

using AllGatherFn = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                                     cudaStream_t);
using ErrorStringFn = const char* (*)(ncclResult_t);

struct NcclSyms {
  AllGatherFn all_gather = nullptr;
  ErrorStringFn error_string = nullptr;
};

static const NcclSyms& nccl_syms() {
  static NcclSyms s;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    void* ag = h ? dlsym(h, "ncclAllGather") : dlsym(RTLD_DEFAULT, "ncclAllGather");
    void* es = h ? dlsym(h, "ncclGetErrorString") : dlsym(RTLD_DEFAULT, "ncclGetErrorString");
    s.all_gather = reinterpret_cast<AllGatherFn>(ag);
    s.error_string = reinterpret_cast<ErrorStringFn>(es);
  });
  return s;
}

}  // namespace dd

extern "C" int dd_scatter_head_shards(const dd_attn_config* cfg, int32_t world, int32_t B,
                                      const void* gathered, void* out, dd_stream_t stream);

extern "C" int dd_allgather_heads(void* nccl_comm, const dd_attn_config* cfg, int32_t world,
                                  int32_t batch_size, const void* local_out, void* gathered,
                                  void* out, dd_stream_t stream) {
  using namespace dd;
  if (!cfg) return fail(DD_ERR_INVALID_ARGUMENT, "config is NULL");
  if (!nccl_comm) return fail(DD_ERR_INVALID_ARGUMENT, "NCCL communicator is NULL");
  if (world <= 0 || cfg->num_kv_heads % world || cfg->num_qo_heads % world)
    return fail(DD_ERR_INVALID_ARGUMENT, "head counts must be divisible by world");
  if (batch_size < 0) return fail(DD_ERR_INVALID_ARGUMENT, "bad batch size");
  if (batch_size == 0) return DD_OK;
  if (!local_out || !gathered || !out) return fail(DD_ERR_INVALID_ARGUMENT, "NULL pointer");
  ncclDataType_t dt;
  if (cfg->q_dtype == DD_DTYPE_BF16) dt = ncclBfloat16;
  else if (cfg->q_dtype == DD_DTYPE_F32) dt = ncclFloat32;
  else return fail(DD_ERR_INVALID_ARGUMENT, "output dtype must be bf16 or f32");
  const NcclSyms& s = nccl_syms();
  if (!s.all_gather) return fail(DD_ERR_NOT_AVAILABLE, "NCCL (libnccl.so.2) is not available");
  const size_t count = (size_t)batch_size * (cfg->num_qo_heads / world) * cfg->head_dim;
  const ncclResult_t r = s.all_gather(local_out, gathered, count, dt,
                                      reinterpret_cast<ncclComm_t>(nccl_comm),
                                      (cudaStream_t)stream);
  if (r != ncclSuccess)
    return fail(DD_ERR_CUDA, std::string("ncclAllGather: ") +
                                 (s.error_string ? s.error_string(r) : std::to_string((int)r)));
  return dd_scatter_head_shards(cfg, world, batch_size, gathered, out, stream);
}
