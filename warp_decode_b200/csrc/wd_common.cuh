// Shared device helpers for the warp_decode_b200 kernels (sm_100a).
//
// * mbarrier / cp.async.bulk (TMA bulk copy, no multicast) wrappers,
// * programmatic-dependent-launch controls,
// * bounded waits (every wait gives up after WD_WAIT_LIMIT_NS and reports
//   WD_STATUS_WAIT_TIMEOUT instead of spinning forever),
// * the per-CTA routing "grouping" that turns the unsorted topk_ids of one
//   call into groups of slots that share an expert, so each expert's weight
//   rows are streamed from HBM once per call instead of once per slot.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "warp_decode.h"

namespace wdb {

// 2 seconds: far above any legitimate wait (a full pipeline stage is a few µs).
constexpr uint64_t WD_WAIT_LIMIT_NS = 2000000000ull;

// Routing limits for the in-CTA grouping.  Calls with more slots are split
// into token chunks on the host.
constexpr int MAX_SLOTS = 512;       // B * topk per launch
constexpr int MAX_DEDUP_E = 1024;    // experts covered by the dedup table
constexpr int GROUP_MAX = 8;         // slots per group (register accumulators)
constexpr int NWARPS = 8;            // compute warps per CTA (both kernels)
#ifndef WD_GU_DEPTH
#define WD_GU_DEPTH 8
#endif
constexpr int GU_DEPTH_MAX = WD_GU_DEPTH;  // gate_up ring slots per consumer warp

// The library-owned status word (one per device context).  The library is
// built as a single translation unit (wd_lib.cu), so the definition lives here.
__device__ uint32_t g_wd_status = 0u;

__device__ __forceinline__ uint32_t* status_ptr(uint32_t* p) {
  return p ? p : &g_wd_status;
}
__device__ __forceinline__ void raise_status(uint32_t* p, uint32_t bits) {
  atomicOr(status_ptr(p), bits);
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false if the
// wait gave up after WD_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 31u) == 0 && globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) return false;
  }
}

// L2 policy for weight streams: every weight byte is read once per call, so
// it is marked evict-first to leave L2 to activations.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D TMA bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch.  Both are no-ops when the grid was launched
// without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Bulk-copy `bytes` (multiple of 16) from global to shared memory in pieces
// of at most 16 KB, all completing on `bar` (expect_tx must cover `bytes`).
__device__ __forceinline__ void bulk_g2s_big(void* dst, const void* src, uint32_t bytes,
                                             uint64_t* bar, uint64_t policy) {
  for (uint32_t off = 0; off < bytes; off += 16384u) {
    const uint32_t len = min(16384u, bytes - off);
    bulk_g2s(static_cast<uint8_t*>(dst) + off, static_cast<const uint8_t*>(src) + off, len, bar,
             policy);
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 16-byte read-only global load (activations: L1-cached, re-read by warps).
__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint4 lds16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// bf16 -> fp32 is exact: a bf16 is the high half of an fp32.
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void unpack_bf16x8(const uint4& v, float (&f)[8]) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}

// a0 += x[0..3] . w[0..3],  a1 += x[4..7] . w[4..7] for 8 packed bf16 pairs,
// with Blackwell's mixed-precision FMA (bf16 inputs, FP32 accumulator).  A
// bf16 widens exactly to FP32 and the product of two bf16 is exact in FP32,
// so each step equals fmaf() on the widened operands: one rounding per FMA.
__device__ __forceinline__ void dot8_bf16(float& a0, float& a1, const uint4& x, const uint4& w) {
  asm("{\n\t"
      ".reg .b16 x0, x1, x2, x3, x4, x5, x6, x7, w0, w1, w2, w3, w4, w5, w6, w7;\n\t"
      "mov.b32 {x0, x1}, %2;\n\tmov.b32 {x2, x3}, %3;\n\t"
      "mov.b32 {x4, x5}, %4;\n\tmov.b32 {x6, x7}, %5;\n\t"
      "mov.b32 {w0, w1}, %6;\n\tmov.b32 {w2, w3}, %7;\n\t"
      "mov.b32 {w4, w5}, %8;\n\tmov.b32 {w6, w7}, %9;\n\t"
      "fma.rn.f32.bf16 %0, x0, w0, %0;\n\tfma.rn.f32.bf16 %1, x4, w4, %1;\n\t"
      "fma.rn.f32.bf16 %0, x1, w1, %0;\n\tfma.rn.f32.bf16 %1, x5, w5, %1;\n\t"
      "fma.rn.f32.bf16 %0, x2, w2, %0;\n\tfma.rn.f32.bf16 %1, x6, w6, %1;\n\t"
      "fma.rn.f32.bf16 %0, x3, w3, %0;\n\tfma.rn.f32.bf16 %1, x7, w7, %1;\n\t"
      "}"
      : "+f"(a0), "+f"(a1)
      : "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w), "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ue8m0 block scale -> 2^(s-127) as fp32 (s = 255 is NaN per OCP MX v1.0).
__device__ __forceinline__ float ue8m0_to_f32(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);  // 2^-127 (fp32 subnormal)
  if (s == 255u) return __uint_as_float(0x7fc00000u);
  return __uint_as_float(s << 23);
}

// The fixed factor of e4m3x16_to_bf16: decoded values are E4M3 x 2^-120.
constexpr float E4M3_BF16_UNSCALE = 0x1p120f;

// Sixteen OCP E4M3 bytes -> sixteen bf16 values in eight packed pairs (byte
// 2j in the low half of p[j]), exact, every value carrying the fixed factor
// 2^-120.  Per byte s.eeee.mmm the bf16 pattern is s at bit 15 and eeee.mmm
// at bits 10..4: an exponent field of e (bias 127 instead of 7, hence the
// 2^-120) with the three mantissa bits on top of bf16's seven, so E4M3
// subnormals (e = 0) land on bf16 subnormals of the same scaled value.  The
// sign-replicating selectors of prmt build [sign x 8 | byte] per 16-bit lane,
// then a shift by 4 and one mask keep sign and magnitude: three integer
// operations per pair, no conversion instructions.  Returns true if some byte
// is an E4M3 NaN (magnitude 0x7f, which would decode to a finite 480 x
// 2^-120): the caller then makes its block scale NaN.  NaN test: x = ~byte &
// 0x7f is 0 exactly for magnitude 0x7f; (x - 1) sets bit 7 of a byte only
// where some byte of the word is 0 (the zero-byte test of Mycroft, 1987).
__device__ __forceinline__ bool e4m3x16_to_bf16(const uint4& v, uint32_t (&p)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t zero_bytes = 0u;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t a, b;
    asm("prmt.b32 %0, %1, 0, 0x9180;" : "=r"(a) : "r"(w[q]));
    asm("prmt.b32 %0, %1, 0, 0xB3A2;" : "=r"(b) : "r"(w[q]));
    p[2 * q] = (a << 4) & 0x87f087f0u;
    p[2 * q + 1] = (b << 4) & 0x87f087f0u;
    zero_bytes |= (~w[q] & 0x7f7f7f7fu) - 0x01010101u;
  }
  return (zero_bytes & 0x80808080u) != 0u;
}

// acc0 += (x[0..7] . w[0..7]) part, acc1 += (x[8..15] . w[8..15]) part, for
// 16 bf16 activations (two 16-byte vectors) against 16 decoded E4M3 weights:
// the same mixed-precision FMA as bf16 weights, on the 2^-120-scaled values.
__device__ __forceinline__ void dot16_e4m3(float& a0, float& a1, const uint4& xa, const uint4& xb,
                                           const uint32_t (&p)[8]) {
  dot8_bf16(a0, a1, xa, make_uint4(p[0], p[1], p[2], p[3]));
  dot8_bf16(a0, a1, xb, make_uint4(p[4], p[5], p[6], p[7]));
}

// One lane's 16-element part of an MX block into the accumulator: the scaled
// sum times 2^120 (exact) times the block scale, or NaN for a NaN byte.
__device__ __forceinline__ float mx_block_fma(float part, uint32_t s, bool nan_byte, float acc) {
  const float sc = nan_byte ? __uint_as_float(0x7fc00000u) : ue8m0_to_f32(s);
  return fmaf(part * E4M3_BF16_UNSCALE, sc, acc);
}

// ---------------------------------------------------------------------------
// Routing groups
// ---------------------------------------------------------------------------
// A group is a set of up to GROUP_MAX slots (flat index b*topk+s) routed to
// the same expert.  With dedup, groups are listed in the order of each
// expert's first appearance in topk_ids, members in increasing slot order, so
// every CTA of a grid derives the identical list (the kernels split work by
// group index).  Without dedup every slot is its own group, in slot order.
// A slot whose expert id is outside [0, E) is always a group of its own with
// expert -1: kernels stream a valid expert's rows for it (keeping the
// pipeline uniform) and give it a zero result.
struct RouteSmem {
  unsigned long long* mask;  // [E+1] tokens routed to each expert (fast path)  (dedup only)
  int* cnt;      // [E+1] slots per expert (entry E: invalid ids)           (dedup only)
  int* off;      // [E+1] first member index of each expert                 (dedup only)
  int* wsum;     // [64]  per-warp partial sums of the scan                 (dedup only)
  int* ids;      // [n]   expert of each slot (validated, -1 if invalid)
  int* rank;     // [n]   position of each slot among its expert's slots
  int* aux;      // [n]   free for the kernels (per-group scratch)
  int* members;  // [n]   slots ordered by (expert, slot); invalid slots last
  int* mtok;     // [n]   token (slot / topk) of each entry of `members`
  int* sg_exp;   // [n]   expert of each capped group (-1: invalid ids)
  int* sg_beg;   // [n]   first member (index into members) of each capped group
  int* sg_cnt;   // [n]   member count of each capped group
  int* nsg;      // [1]   number of capped groups
};

// Shared-memory bytes needed by RouteSmem for n slots and E experts.  The
// base must be 8-byte aligned.
__host__ __device__ inline int route_smem_bytes(int n, int E, bool dedup) {
  int ints = 8 * n + 1 + (dedup ? 4 * (E + 1) + 64 : 0);
  return ((ints * 4 + 127) / 128) * 128;
}

__device__ inline RouteSmem route_carve(int* base, int n, int E, bool dedup) {
  RouteSmem r;
  int* p = base;
  r.mask = dedup ? reinterpret_cast<unsigned long long*>(p) : nullptr;
  p += dedup ? 2 * (E + 1) : 0;
  r.cnt = dedup ? p : nullptr; p += dedup ? E + 1 : 0;
  r.off = dedup ? p : nullptr; p += dedup ? E + 1 : 0;
  r.wsum = dedup ? p : nullptr; p += dedup ? 64 : 0;
  r.ids = p; p += n;
  r.rank = p; p += n;
  r.aux = p; p += n;
  r.members = p; p += n;
  r.mtok = p; p += n;
  r.sg_exp = p; p += n;
  r.sg_beg = p; p += n;
  r.sg_cnt = p; p += n;
  r.nsg = p;
  return r;
}

struct NoInit {
  __device__ void operator()() const {}
};

// Routing of one launch, computed by every CTA (all threads; ends with
// __syncthreads).  Validates topk_ids (out-of-range ids become -1 and raise
// WD_STATUS_BAD_EXPERT_ID), then groups the slots by expert:
//  * dedup: one group per touched expert (for n <= 64 in the order of first
//    appearance, found by one warp; else in ascending expert id), members
//    in slot order, split into groups of at most `cap` members; all invalid
//    slots form one group with expert -1.  For n > 64 a stable counting sort:
//    with at most 64 tokens and no expert repeated inside a token, each
//    expert's 64-bit token mask (shared-memory atomicOr) gives every slot
//    its rank directly; otherwise one warp ranks the slots 32 at a time
//    (match_any).  One block-wide scan places the experts.  Same result in
//    every CTA: deterministic.
//  * no dedup: every slot is its own group (slot order).
// `scale` (optional, n floats) is copied to `s_scale` in the same global
// round trip as the ids.  `init` runs after the loads are issued and before
// they are used, so a caller's own set-up overlaps their latency.
// The grouping follows the outputs-not-experts idea of the reference (no
// align/permute pass over unsorted topk_ids, csrc/moe_gate_up_3d_batched.cu)
// but shares each expert's weight stream between the slots routed to it.
// kMode: ROUTE_ANY, ROUTE_SMALL (the caller guarantees n <= 64 and
// blockDim.x >= 64: only the one-warp grouping is compiled) or ROUTE_LARGE
// (n > 64: the one-warp grouping is left out).  Less code to fetch on a
// launch's cold start.
enum RouteMode : int { ROUTE_ANY = 0, ROUTE_SMALL = 1, ROUTE_LARGE = 2 };
template <bool kScale = false, class Init = NoInit, int kMode = ROUTE_ANY>
__device__ inline void route_build(const RouteSmem& r, const int32_t* __restrict__ topk_ids,
                                   int n, int E, int K, bool dedup, int cap, uint32_t* status,
                                   Init init = Init(), const float* __restrict__ scale = nullptr,
                                   float* s_scale = nullptr) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5;
  // slots per thread (blockDim >= 128, or >= 64 with ROUTE_SMALL)
  constexpr bool kSmall = kMode == ROUTE_SMALL;
  constexpr int PER = kSmall ? 1 : (MAX_SLOTS + 127) / 128;
  constexpr int SPER = kScale ? PER : 1;
  int ev[PER];
  float sv[SPER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = tid + k * nt;
    ev[k] = i < n ? __ldg(topk_ids + i) : 0;
    if constexpr (kScale) sv[k] = i < n ? __ldg(scale + i) : 0.f;
  }
  init();
  if (!kSmall && dedup) {
    for (int e = tid; e <= E; e += nt) {
      r.mask[e] = 0ull;
      r.cnt[e] = 0;
    }
  }
  bool bad = false;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = tid + k * nt;
    if (i < n) {
      int e = ev[k];
      if (e < 0 || e >= E) { e = -1; bad = true; }
      r.ids[i] = e;
      if constexpr (kScale) s_scale[i] = sv[k];
    }
  }
  if (__syncthreads_or(bad) && tid == 0) raise_status(status, WD_STATUS_BAD_EXPERT_ID);
  if (!dedup) {
    for (int i = tid; i < n; i += nt) {
      r.sg_exp[i] = r.ids[i];
      r.sg_beg[i] = i;
      r.sg_cnt[i] = 1;
      r.members[i] = i;
      r.mtok[i] = i / K;
    }
    if (tid == 0) *r.nsg = n;
    __syncthreads();
    return;
  }
  if (kMode != ROUTE_LARGE && (kSmall || n <= 64)) {
    // Small launch: one warp groups all slots (first-appearance order of
    // the experts, members in slot order) with shared-memory atomics on the
    // touched buckets only and ballot/shuffle scans: one block barrier.
    if (warp == 0) {
      int* first = reinterpret_cast<int*>(r.mask);  // [E+1] first slot of each bucket
      int* c0 = r.cnt;                              // [E+1] slots in 0..31
      int* c1 = r.off;                              // [E+1] slots in 32..63
      const int i0 = lane, i1 = lane + 32;
      const bool v0 = i0 < n, v1 = i1 < n;
      const int k0 = v0 ? (r.ids[i0] < 0 ? E : r.ids[i0]) : -1;
      const int k1 = v1 ? (r.ids[i1] < 0 ? E : r.ids[i1]) : -1;
      if (v0) { first[k0] = 0x7fffffff; c0[k0] = 0; c1[k0] = 0; }
      if (v1) { first[k1] = 0x7fffffff; c0[k1] = 0; c1[k1] = 0; }
      __syncwarp();
      if (v0) { atomicMin(&first[k0], i0); atomicAdd(&c0[k0], 1); }
      if (v1) { atomicMin(&first[k1], i1); atomicAdd(&c1[k1], 1); }
      __syncwarp();
      const unsigned lt = (1u << lane) - 1u;
      const unsigned m0 = __match_any_sync(0xffffffffu, v0 ? k0 : -2 - lane);
      const unsigned m1 = __match_any_sync(0xffffffffu, v1 ? k1 : -2 - lane);
      const int rank0 = __popc(m0 & lt);
      const int rank1 = (v1 ? c0[k1] : 0) + __popc(m1 & lt);
      const bool f0 = v0 && first[k0] == i0, f1 = v1 && first[k1] == i1;
      const int sz0 = f0 ? c0[k0] + c1[k0] : 0, sz1 = f1 ? c0[k1] + c1[k1] : 0;
      const int ns0 = (sz0 + cap - 1) / cap, ns1 = (sz1 + cap - 1) / cap;
      // Exclusive scans in group (= slot) order of sizes and subgroup counts.
      int a0 = sz0, a1 = sz1, s0 = ns0, s1 = ns1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t0 = __shfl_up_sync(0xffffffffu, a0, o), t1 = __shfl_up_sync(0xffffffffu, a1, o);
        const int u0 = __shfl_up_sync(0xffffffffu, s0, o), u1 = __shfl_up_sync(0xffffffffu, s1, o);
        if (lane >= o) { a0 += t0; a1 += t1; s0 += u0; s1 += u1; }
      }
      const int tot_a0 = __shfl_sync(0xffffffffu, a0, 31), tot_s0 = __shfl_sync(0xffffffffu, s0, 31);
      const int off0 = a0 - sz0, off1 = tot_a0 + a1 - sz1;      // member offset of the group
      const int so0 = s0 - ns0, so1 = tot_s0 + s1 - ns1;        // first subgroup of the group
      if (lane == 31) *r.nsg = tot_s0 + s1;
      if (f0)
        for (int j = 0; j < ns0; ++j) {
          r.sg_exp[so0 + j] = k0 < E ? k0 : -1;
          r.sg_beg[so0 + j] = off0 + j * cap;
          r.sg_cnt[so0 + j] = min(cap, sz0 - j * cap);
        }
      if (f1)
        for (int j = 0; j < ns1; ++j) {
          r.sg_exp[so1 + j] = k1 < E ? k1 : -1;
          r.sg_beg[so1 + j] = off1 + j * cap;
          r.sg_cnt[so1 + j] = min(cap, sz1 - j * cap);
        }
      // Member position = offset of the slot's group + its rank: the group's
      // offset lives in the lane of the group's first slot.
      const int fs0 = v0 ? first[k0] : 0, fs1 = v1 ? first[k1] : 0;
      const int o00 = __shfl_sync(0xffffffffu, off0, fs0 & 31), o01 = __shfl_sync(0xffffffffu, off1, fs0 & 31);
      const int o10 = __shfl_sync(0xffffffffu, off0, fs1 & 31), o11 = __shfl_sync(0xffffffffu, off1, fs1 & 31);
      if (v0) {
        const int p = (fs0 < 32 ? o00 : o01) + rank0;
        r.members[p] = i0;
        r.mtok[p] = i0 / K;
      }
      if (v1) {
        const int p = (fs1 < 32 ? o10 : o11) + rank1;
        r.members[p] = i1;
        r.mtok[p] = i1 / K;
      }
    }
    __syncthreads();
    return;
  }
  if constexpr (kSmall) return;  // not reached: n <= 64
  // Token masks; an expert (or the invalid bucket) twice in one token, or
  // more than 64 tokens, sends the launch to the ordered warp pass.
  const int ntok = n / K;
  bool slow = ntok > 64;
  if (!slow && (32 % K) == 0) {
    // K divides 32: a warp's 32 consecutive slots are whole tokens, so one
    // match_any on (expert, token) finds a repeat inside a token.  The mask
    // bit goes in with a 32-bit shared atomic on the word holding it.
    for (int c = warp * 32; c < n; c += nt) {
      const int i = c + lane;
      const bool v = i < n;
      const int key = v ? (r.ids[i] < 0 ? E : r.ids[i]) : 0;
      const int t = i / K;
      const unsigned m = __match_any_sync(0xffffffffu, v ? key * 64 + t : -1 - lane);
      slow |= __popc(m) > 1;
      if (v)
        atomicOr(reinterpret_cast<unsigned*>(&r.mask[key]) + (t >> 5), 1u << (t & 31));
    }
  } else if (!slow) {
    for (int i = tid; i < n; i += nt) {
      const int key = r.ids[i] < 0 ? E : r.ids[i];
      const int t = i / K;
      for (int j = t * K; j < i; ++j) slow |= ((r.ids[j] < 0 ? E : r.ids[j]) == key);
      atomicOr(reinterpret_cast<unsigned*>(&r.mask[key]) + (t >> 5), 1u << (t & 31));
    }
  }
  slow = __syncthreads_or(slow);
  if (!slow) {
    for (int i = tid; i < n; i += nt) {
      const int key = r.ids[i] < 0 ? E : r.ids[i];
      const int t = i / K;
      r.rank[i] = __popcll(r.mask[key] & ((1ull << t) - 1ull));
    }
    for (int e = tid; e <= E; e += nt) r.cnt[e] = __popcll(r.mask[e]);
  } else if (warp == 0) {
    // Stable rank within each expert, 32 slots at a time.
    for (int c = 0; c < n; c += 32) {
      const int i = c + lane;
      const bool v = i < n;
      const int key = v ? (r.ids[i] < 0 ? E : r.ids[i]) : E + 1 + lane;
      const unsigned m = __match_any_sync(0xffffffffu, key);
      const int base = v ? r.cnt[key] : 0;
      __syncwarp();
      if (v) {
        r.rank[i] = base + __popc(m & ((1u << lane) - 1u));
        if (lane == __ffs(m) - 1) r.cnt[key] = base + __popc(m);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  // Exclusive scans over the E + 1 buckets: member offsets and capped-group
  // indices, each thread owning a contiguous run of buckets.
  const int NE = E + 1;
  const int per = (NE + nt - 1) / nt;
  const int e0 = min(NE, tid * per), e1 = min(NE, e0 + per);
  int sc = 0, ss = 0;
  for (int e = e0; e < e1; ++e) {
    const int c = r.cnt[e];
    sc += c;
    ss += (c + cap - 1) / cap;
  }
  int ic = sc, is = ss;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t1 = __shfl_up_sync(0xffffffffu, ic, o);
    const int t2 = __shfl_up_sync(0xffffffffu, is, o);
    if (lane >= o) { ic += t1; is += t2; }
  }
  if (lane == 31) { r.wsum[2 * warp] = ic; r.wsum[2 * warp + 1] = is; }
  __syncthreads();
  int oc = ic - sc, os = is - ss;
  for (int w = 0; w < warp; ++w) { oc += r.wsum[2 * w]; os += r.wsum[2 * w + 1]; }
  for (int e = e0; e < e1; ++e) {
    const int c = r.cnt[e];
    r.off[e] = oc;
    for (int j = 0; j * cap < c; ++j) {
      r.sg_exp[os] = e < E ? e : -1;
      r.sg_beg[os] = oc + j * cap;
      r.sg_cnt[os] = min(cap, c - j * cap);
      ++os;
    }
    oc += c;
  }
  if (tid == nt - 1) *r.nsg = os;
  __syncthreads();
  for (int i = tid; i < n; i += nt) {
    const int e = r.ids[i];
    const int p = r.off[e < 0 ? E : e] + r.rank[i];
    r.members[p] = i;
    r.mtok[p] = i / K;
  }
  __syncthreads();
}

// Grid-scope counter accesses (grid barriers inside one launch) and L2 loads.
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add_u64(unsigned long long* p,
                                                        unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// 16-byte load through L2 only (data written by other CTAs of this grid).
__device__ __forceinline__ uint4 ldcg16(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
// Grid barriers of the single-launch kernels share one 64-bit counter (the
// caller's `sync` words, or the library's): every launch adds exactly
// GRID_BAR_UNITS in total, CTA c of G its share (c + 1) U / G - c U / G, so
// between launches the counter is a multiple of U whatever grid each launch
// used, and a CTA that reads the counter before adding its own share knows
// the value that ends the barrier.  A CTA adds its share before it waits,
// also on its abort paths, so the invariant survives a timed-out call.
constexpr unsigned long long GRID_BAR_UNITS = 4096;  // >= every grid of the library
__device__ __forceinline__ unsigned long long grid_bar_share() {
  const unsigned long long c = blockIdx.x, G = gridDim.x;
  return (c + 1) * GRID_BAR_UNITS / G - c * GRID_BAR_UNITS / G;
}
__device__ __forceinline__ unsigned long long grid_bar_target(unsigned long long at_entry) {
  return (at_entry / GRID_BAR_UNITS + 1) * GRID_BAR_UNITS;
}

// System-scope release store / acquire load (flags shared with peer GPUs).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Non-blocking mbarrier phase test.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

}  // namespace wdb
