// TEST INFRASTRUCTURE ONLY: C entry points over the reference's own kernel
// launchers, so tests can run Religious-J/warp_decode's CUDA kernels (rebuilt
// unmodified for sm_100a by oracle/Makefile) next to ours on the same box.
//
// The launchers are declared exactly as the reference binding declares them
// (csrc/binding.cpp:6-25 of the reference); their definitions come from the
// reference sources compiled by the Makefile.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace warp_decode {
void launch_moe_gate_up_3d_batched(const __nv_bfloat16* X, const __nv_bfloat16* W,
                                   const int* topk_ids, __nv_bfloat16* out, int B, int E,
                                   int topk, int hidden, int inter, cudaStream_t stream);
void launch_moe_down_3d_batched(const __nv_bfloat16* buffer, const __nv_bfloat16* W,
                                const int* topk_ids, const float* topk_scale,
                                __nv_bfloat16* out, int B, int E, int topk, int hidden,
                                int inter, cudaStream_t stream);
}  // namespace warp_decode

extern "C" {

__attribute__((visibility("default"))) int wdref_gate_up(const void* x, const void* w,
                                                         const int* ids, void* out, int B, int E,
                                                         int topk, int hidden, int inter,
                                                         void* stream) {
  warp_decode::launch_moe_gate_up_3d_batched(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), ids,
      static_cast<__nv_bfloat16*>(out), B, E, topk, hidden, inter,
      static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

__attribute__((visibility("default"))) int wdref_down(const void* buffer, const void* w,
                                                      const int* ids, const float* scale,
                                                      void* out, int B, int E, int topk,
                                                      int hidden, int inter, void* stream) {
  warp_decode::launch_moe_down_3d_batched(
      static_cast<const __nv_bfloat16*>(buffer), static_cast<const __nv_bfloat16*>(w), ids,
      scale, static_cast<__nv_bfloat16*>(out), B, E, topk, hidden, inter,
      static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
