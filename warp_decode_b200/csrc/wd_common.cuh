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
// the same expert.  Groups are listed in the order of each expert's first
// appearance in topk_ids, members in increasing slot order, so every CTA of a
// grid derives the identical list (the kernels split work by group index).
// An expert id outside [0, E) is mapped to the expert value -1 (such groups
// are never used to address weights).
struct RouteSmem {
  int* ids;      // [n]   expert of each slot (validated, -1 if invalid)
  int* tab;      // [E+1] dedup table (min slot index, later -(rank+1));
                 //       entry E collects the invalid ids
  int* cnt;      // [n]   members per expert group, later exclusive offsets
  int* gexp;     // [n]   expert of each expert group
  int* rankpos;  // [n]   rank << 12 | position within group
  int* members;  // [n]   slots ordered by (group, slot)
  int* sg_exp;   // [n]   expert of each capped group (or -1)
  int* sg_beg;   // [n]   first member (index into members) of each capped group
  int* sg_cnt;   // [n]   member count of each capped group
  int* nsg;      // [1]   number of capped groups
};

// Shared-memory bytes needed by RouteSmem for n slots and E experts.
__host__ __device__ inline int route_smem_bytes(int n, int E, bool dedup) {
  int ints = 9 * n + 1 + (dedup ? E + 1 : 0);
  return ((ints * 4 + 127) / 128) * 128;
}

__device__ inline RouteSmem route_carve(int* base, int n, int E, bool dedup) {
  RouteSmem r;
  r.ids = base;
  r.cnt = r.ids + n;
  r.gexp = r.cnt + n;
  r.rankpos = r.gexp + n;
  r.members = r.rankpos + n;
  r.sg_exp = r.members + n;
  r.sg_beg = r.sg_exp + n;
  r.sg_cnt = r.sg_beg + n;
  r.nsg = r.sg_cnt + n;
  r.tab = dedup ? r.nsg + 1 : nullptr;
  return r;
}

// Build the groups for slots [0, n) of `topk_ids` (a device pointer).
// Must be called by all threads of the CTA; ends with __syncthreads().
// dedup = false makes every slot its own group (no table, no scans).
__device__ inline void build_groups(const RouteSmem& r, const int32_t* __restrict__ topk_ids,
                                    int n, int E, bool dedup, uint32_t* status) {
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  bool bad = false;
  for (int i = tid; i < n; i += nthreads) {
    int e = __ldg(topk_ids + i);
    if (e < 0 || e >= E) { e = -1; bad = true; }
    r.ids[i] = e;
  }
  if (__syncthreads_or(bad) && tid == 0) raise_status(status, WD_STATUS_BAD_EXPERT_ID);

  if (!dedup) {
    for (int i = tid; i < n; i += nthreads) {
      r.members[i] = i;
      r.sg_exp[i] = r.ids[i];
      r.sg_beg[i] = i;
      r.sg_cnt[i] = 1;
    }
    if (tid == 0) *r.nsg = n;
    __syncthreads();
    return;
  }

  // Invalid ids all go to one pseudo-expert E (table slot E).
  for (int e = tid; e <= E; e += nthreads) r.tab[e] = 0x7fffffff;
  for (int i = tid; i < n; i += nthreads) r.cnt[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += nthreads) {
    const int e = r.ids[i];
    atomicMin(&r.tab[e < 0 ? E : e], i);
  }
  __syncthreads();

  // One warp walks the slots in order: assign group ranks (order of first
  // appearance) and each slot's position inside its group.  Deterministic.
  if (tid < 32) {
    const int lane = tid;
    const unsigned lt = (1u << lane) - 1u;
    int base = 0;
    for (int c = 0; c < n; c += 32) {
      const int i = c + lane;
      const bool valid = i < n;
      const int e = valid ? r.ids[i] : 0;
      const int key = e < 0 ? E : e;
      const int t = valid ? r.tab[key] : 0;
      const bool first = valid && (t == i);
      const unsigned fb = __ballot_sync(0xffffffffu, first);
      int rank = base + __popc(fb & lt);
      // Non-first slot: its group was opened earlier (t < 0 after rewrite),
      // or by a lane of this same chunk (t = that lane's slot index).
      const int src_lane = (valid && t >= 0) ? (t - c) : lane;
      const int lane_rank = __shfl_sync(0xffffffffu, rank, src_lane & 31);
      if (valid && !first) rank = (t < 0) ? (-t - 1) : lane_rank;
      // Position inside the group: earlier chunks (cnt) + earlier lanes here.
      const unsigned same = __match_any_sync(0xffffffffu, valid ? rank : -1);
      const int pos = valid ? (r.cnt[rank] + __popc(same & lt)) : 0;
      __syncwarp();
      if (valid) {
        r.rankpos[i] = (rank << 12) | pos;
        if ((same & lt) == 0u) r.cnt[rank] += __popc(same);
        if (first) { r.tab[key] = -(rank + 1); r.gexp[rank] = e; }
      }
      __syncwarp();
      base += __popc(fb);
    }
    // Exclusive offsets of expert groups and the capped-group list.
    int off = 0, sg = 0;
    for (int c = 0; c < base; c += 32) {
      const int g = c + lane;
      const int cnt = g < base ? r.cnt[g] : 0;
      const int nsub = (cnt + GROUP_MAX - 1) / GROUP_MAX;
      int inc_cnt = cnt, inc_sub = nsub;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc_cnt, o);
        const int b = __shfl_up_sync(0xffffffffu, inc_sub, o);
        if (lane >= o) { inc_cnt += a; inc_sub += b; }
      }
      const int my_off = off + inc_cnt - cnt;
      const int my_sg = sg + inc_sub - nsub;
      if (g < base) {
        r.cnt[g] = my_off;  // now the exclusive member offset of group g
        const int e = r.gexp[g];
        for (int j = 0; j < nsub; ++j) {
          r.sg_exp[my_sg + j] = e;
          r.sg_beg[my_sg + j] = my_off + j * GROUP_MAX;
          r.sg_cnt[my_sg + j] = min(GROUP_MAX, cnt - j * GROUP_MAX);
        }
      }
      off += __shfl_sync(0xffffffffu, inc_cnt, 31);
      sg += __shfl_sync(0xffffffffu, inc_sub, 31);
    }
    if (lane == 0) *r.nsg = sg;
  }
  __syncthreads();
  for (int i = tid; i < n; i += nthreads) {
    const int rp = r.rankpos[i];
    r.members[r.cnt[rp >> 12] + (rp & 0xfff)] = i;
  }
  __syncthreads();
}

}  // namespace wdb
