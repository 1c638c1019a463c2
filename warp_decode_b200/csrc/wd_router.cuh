// Router producer for the MoE FFN, sm_100a: top-k expert selection and the
// routing weights from router logits.  Upstream of the two kernels (it makes
// their topk_ids / topk_scale); the reference has no router and takes both as
// inputs (csrc/binding.cpp:79-121).
//
//   topk_ids[b, :]    = the k largest logits[b, :], in descending order; equal
//                       logits in ascending expert order (deterministic)
//   topk_weights[b,:] = renormalize ? softmax over the k selected logits
//                                   : softmax over all E logits, at the k ids
//
// One warp per token: every lane keeps its strided share of the token's row
// in registers (E <= 32 * ROUTER_PER) and the warp extracts the maximum k
// times (lane-local scan over the entries not yet taken, then a 5-step
// shuffle argmax on (value, index)).
// HBM-trivial (B * E logits); one launch of ceil(B / 8) CTAs of 256 threads.
#pragma once

#include "wd_common.cuh"

namespace wdb {

constexpr int ROUTER_PER = 32;     // logits per lane: E <= 1024
constexpr int ROUTER_MAX_K = 32;
constexpr int ROUTER_WARPS = 8;

struct RouterArgs {
  const void* logits;  // [B, E] bf16 or fp32
  int logits_fp32;
  int32_t* ids;        // [B, K]
  float* weights;      // [B, K]
  int B, E, K;
  int renormalize;
};

// (v, i) beats (w, j): larger value, then smaller index.  NaN logits never win.
__device__ __forceinline__ bool router_better(float v, int i, float w, int j) {
  return v > w || (v == w && i < j);
}

__global__ void __launch_bounds__(ROUTER_WARPS * 32) moe_router_topk_kernel(const RouterArgs a) {
  const int lane = threadIdx.x & 31;
  const int b = (int)blockIdx.x * ROUTER_WARPS + (threadIdx.x >> 5);
  if (b >= a.B) return;  // whole warps leave together
  const int E = a.E;
  float v[ROUTER_PER];
#pragma unroll
  for (int q = 0; q < ROUTER_PER; ++q) {
    const int e = lane + 32 * q;
    float x = -INFINITY;
    if (e < E) {
      if (a.logits_fp32)
        x = reinterpret_cast<const float*>(a.logits)[(size_t)b * E + e];
      else
        x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.logits)[(size_t)b * E + e]);
      if (x != x) x = -INFINITY;  // NaN: never selected before a number
    }
    v[q] = x;
  }
  float sel_v = 0.f;  // lane k keeps the k-th selected logit
  int sel_i = 0;
  uint32_t taken = 0u;  // bit q: this lane's entry q already selected
  for (int k = 0; k < a.K; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < ROUTER_PER; ++q) {
      const int e = lane + 32 * q;
      if (e < E && !((taken >> q) & 1u) && router_better(v[q], e, bv, bi)) {
        bv = v[q];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (router_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // mark the winner taken in its owner lane (a flag, not a -inf value:
    // -inf is a legal logit)
    if (lane == (bi & 31)) taken |= 1u << (bi >> 5);
    if (lane == k) {
      sel_v = bv;
      sel_i = bi;
    }
  }
  // Weights: exp(l - max) over the selected (renormalised) or over all E;
  // the largest logit is the first selected one.
  float ref = __shfl_sync(0xffffffffu, sel_v, 0);
  if (!(ref > -INFINITY)) ref = 0.f;  // every logit -inf (or NaN)
  float den = 0.f;
  if (a.renormalize) {
    den = lane < a.K ? expf(sel_v - ref) : 0.f;
  } else {
#pragma unroll
    for (int q = 0; q < ROUTER_PER; ++q) den += (v[q] == -INFINITY) ? 0.f : expf(v[q] - ref);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  if (lane < a.K) {
    a.ids[(size_t)b * a.K + lane] = sel_i;
    // den = 0 only if every logit is -inf (or NaN): uniform weights then
    a.weights[(size_t)b * a.K + lane] = den > 0.f ? expf(sel_v - ref) / den : 1.f / (float)a.K;
  }
}

}  // namespace wdb
