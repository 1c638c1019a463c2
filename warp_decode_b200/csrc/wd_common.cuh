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
#define WD_GU_DEPTH 2
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
  int* ids;      // [n]   expert of each slot (validated, -1 if invalid)
  int* tab;      // [E]   dedup table: min slot index, then group rank
  int* aux;      // [n]   scratch
  int* rank;     // [n]   group rank of each slot
  int* gcnt;     // [n]   members per group
  int* goff;     // [n]   first member index of each group
  int* members;  // [n]   slots ordered by (group, slot)
  int* mtok;     // [n]   token (slot / topk) of each entry of `members`
  int* sg_exp;   // [n]   expert of each capped group (-1: invalid slot)
  int* sg_beg;   // [n]   first member (index into members) of each capped group
  int* sg_cnt;   // [n]   member count of each capped group
  int* nsg;      // [1]   number of capped groups
};

// Shared-memory bytes needed by RouteSmem for n slots and E experts.
__host__ __device__ inline int route_smem_bytes(int n, int E, bool dedup) {
  int ints = 11 * n + 1 + (dedup ? E : 0);
  return ((ints * 4 + 127) / 128) * 128;
}

__device__ inline RouteSmem route_carve(int* base, int n, int E, bool dedup) {
  RouteSmem r;
  int* p = base;
  r.ids = p; p += n;
  r.aux = p; p += n;
  r.rank = p; p += n;
  r.gcnt = p; p += n;
  r.goff = p; p += n;
  r.members = p; p += n;
  r.mtok = p; p += n;
  r.sg_exp = p; p += n;
  r.sg_beg = p; p += n;
  r.sg_cnt = p; p += n;
  r.nsg = p; p += 1;
  r.tab = dedup ? p : nullptr;
  return r;
}

// Exclusive prefix sum of a[0..cnt) in place by one warp (lanes in step);
// returns the total.  cnt <= MAX_SLOTS.
__device__ __forceinline__ int warp_exclusive_scan(int* a, int cnt, int lane) {
  int base = 0;
  for (int c = 0; c < cnt; c += 32) {
    const int i = c + lane;
    const int v = i < cnt ? a[i] : 0;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    if (i < cnt) a[i] = base + inc - v;
    base += __shfl_sync(0xffffffffu, inc, 31);
  }
  return base;
}

// Load and validate this launch's topk_ids into shared memory.  All threads.
// Ends with __syncthreads().
__device__ inline void load_ids(const RouteSmem& r, const int32_t* __restrict__ topk_ids, int n,
                                int E, uint32_t* status) {
  bool bad = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int e = __ldg(topk_ids + i);
    if (e < 0 || e >= E) { e = -1; bad = true; }
    r.ids[i] = e;
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) raise_status(status, WD_STATUS_BAD_EXPERT_ID);
}

// Build the capped groups from r.ids (see load_ids).  All threads; ends with
// __syncthreads().
__device__ inline void build_groups(const RouteSmem& r, int n, int E, int K, bool dedup,
                                    int cap = GROUP_MAX) {
  const int tid = threadIdx.x;
  const int nt = blockDim.x;
  const int lane = tid & 31;
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
  __shared__ int s_groups;
  for (int e = tid; e < E; e += nt) r.tab[e] = 0x7fffffff;
  for (int i = tid; i < n; i += nt) r.gcnt[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += nt) {
    const int e = r.ids[i];
    if (e >= 0) atomicMin(&r.tab[e], i);
  }
  __syncthreads();
  // A group opens at the first slot of each expert and at every invalid slot.
  for (int i = tid; i < n; i += nt) {
    const int e = r.ids[i];
    const int open = (e < 0 || r.tab[e] == i) ? 1 : 0;
    r.aux[i] = open;
    r.rank[i] = open;
  }
  __syncthreads();
  if (tid < 32) {
    const int groups = warp_exclusive_scan(r.rank, n, lane);  // rank of opening slots
    if (lane == 0) s_groups = groups;
  }
  __syncthreads();
  for (int i = tid; i < n; i += nt) {
    if (r.aux[i]) {
      const int e = r.ids[i];
      if (e >= 0) r.tab[e] = r.rank[i];
    }
  }
  __syncthreads();
  // Every slot learns its group; counts and (unordered) positions by atomics.
  for (int i = tid; i < n; i += nt) {
    const int e = r.ids[i];
    const int g = (e < 0) ? r.rank[i] : r.tab[e];
    r.rank[i] = g;
    r.aux[i] = atomicAdd(&r.gcnt[g], 1);
  }
  __syncthreads();
  const int groups = s_groups;
  if (tid < 32) {
    for (int g = lane; g < groups; g += 32) r.goff[g] = r.gcnt[g];
    __syncwarp();
    warp_exclusive_scan(r.goff, groups, lane);
  }
  __syncthreads();
  for (int i = tid; i < n; i += nt) r.members[r.goff[r.rank[i]] + r.aux[i]] = i;
  __syncthreads();
  // Members in slot order (groups are small: insertion sort per group), and
  // the number of capped groups per group.
  for (int g = tid; g < groups; g += nt) {
    const int b = r.goff[g], c = r.gcnt[g];
    for (int x = b + 1; x < b + c; ++x) {
      const int v = r.members[x];
      int y = x - 1;
      while (y >= b && r.members[y] > v) { r.members[y + 1] = r.members[y]; --y; }
      r.members[y + 1] = v;
    }
    r.aux[g] = (c + cap - 1) / cap;
  }
  __syncthreads();
  if (tid < 32) {
    const int total = warp_exclusive_scan(r.aux, groups, lane);
    if (lane == 0) *r.nsg = total;
  }
  __syncthreads();
  for (int g = tid; g < groups; g += nt) {
    const int b = r.goff[g], c = r.gcnt[g], s0 = r.aux[g];
    const int e = r.ids[r.members[b]];
    for (int j = 0; j * cap < c; ++j) {
      r.sg_exp[s0 + j] = e;
      r.sg_beg[s0 + j] = b + j * cap;
      r.sg_cnt[s0 + j] = min(cap, c - j * cap);
    }
  }
  for (int i = tid; i < n; i += nt) r.mtok[i] = r.members[i] / K;
  __syncthreads();
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
