// Launch accounting / profiling hooks (profile.cu). Kind indices are the
// ones reported by dd_profile_read.
#pragma once
#include <cuda_runtime.h>

namespace dd {
enum ProfKind {
  kProfSimple = 0,  // attn_simple_kernel
  kProfMma = 1,     // attn_mma_kernel
  kProfTc = 2,      // tcgen05 attention kernel
  kProfMerge = 3,   // merge_paths_kernel / merge_two_kernel
  kProfQuant = 4,   // quantize / dequantize kernels
  kProfOther = 5,   // append, scatter
  kNumProf = 6
};
void prof_begin(int kind, cudaStream_t st);
void prof_end(int kind, cudaStream_t st);
// True while per-launch timing is on: launches then run one at a time on
// the caller's stream, so each event pair brackets one kernel alone.
bool prof_timing_on();

// RAII bracket around one launch.
struct ProfScope {
  int kind;
  cudaStream_t st;
  ProfScope(int k, cudaStream_t s) : kind(k), st(s) { prof_begin(k, s); }
  ~ProfScope() { prof_end(kind, st); }
};
}  // namespace dd
