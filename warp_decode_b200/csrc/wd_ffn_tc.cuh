// The whole MoE FFN in ONE launch on the tcgen05 tensor cores, sm_100a:
//   phase 1  h = silu(x . Wg) * (x . Wu)   (the body of moe_gate_up_tc_kernel;
//            csrc/moe_gate_up_3d_batched.cu:49-115 of the reference)
//   phase 2  y = sum_s scale_s * (h_s . Wd)  (the body of moe_down_tc_kernel;
//            csrc/moe_down_3d_batched.cu:45-122)
// for the batches where the two tensor-core kernels run (more routed slots
// than the SIMT single launch takes).
//
// Why: as two launches, the down kernel starts only after the last gate_up
// CTA has exited and then spends the launch gap, its routing and its first
// weight round trip before its first MMA, with HBM idle.  Here:
//  * the routing is computed once, at entry, for both phases (the down
//    phase's items are the gate_up groups cut into runs of DTC_N members);
//  * TMEM is allocated once (128 columns cover both phases);
//  * a CTA that has finished its gate_up items adds its share to the grid
//    barrier and starts the down phase at once: its weight producer streams
//    the first down stages while other CTAs still finish gate_up, and only
//    the gather warps wait for the barrier (h of the whole launch) before
//    reading h through L2.
// Grid: the down phase's clusters (ceil(H / 128) row tiles x CL CTAs), all
// co-resident (cooperative launch); gate_up runs on the same CTAs, each CTA
// taking whole items or, where items are few for the grid, 1/CL of K of its
// cluster's items (the split K of moe_gate_up_tc_kernel).
// Shared memory: the routing region (kept for the whole launch) followed by
// one phase region that each phase carves in turn; the gate_up phase
// invalidates its mbarriers before the down phase initialises its own.
#pragma once

#include "wd_down_tc.cuh"
#include "wd_gate_up_tc.cuh"

namespace wdb {

struct FfnTcArgs {
  GateUpTcArgs gu;          // phase 1 (cl = 1, or the launch's cluster size: split K)
  DownTcArgs dn;            // phase 2 (cl = the launch's cluster size)
  const int32_t* ids;       // [B, K]
  const float* scale;       // [B, K]
  unsigned long long* sync; // grid-barrier counter (GRID_BAR_UNITS per launch)
  int B, E, K;
  int route_bytes;          // bytes of the routing region (multiple of 1024)
};

constexpr int FFN_TC_TMEM_COLS = 128;  // gate_up: 2 x 64 columns; down: 4 x 16

// Routing region: RouteSmem of the call, the top-k weights, and the down
// phase's item table [3][n] + count.
__host__ __device__ inline int ffn_tc_route_bytes(int n, int E) {
  const int b = route_smem_bytes(n, E, true) + 4 * n + 4 * (3 * n + 1);
  return (b + 1023) / 1024 * 1024;
}

// kTP: the down phase ends in the fused all-reduce of the tensor-core down
// kernel (fa.dn.tp: y = bf16 sum over the group's ranks).
template <int kRoute, bool kTP = false>
__global__ void __launch_bounds__(DTC_THREADS, 1)
    moe_ffn_tc_kernel(const __grid_constant__ CUtensorMap tm_gw,
                      const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_dw, const FfnTcArgs fa) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long sync0;
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = smem_raw + pad;
  const int n = fa.B * fa.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const RouteSmem r = route_carve(reinterpret_cast<int*>(base), n, fa.E, true);
  float* s_scale = reinterpret_cast<float*>(base + route_smem_bytes(n, fa.E, true));
  int* dsg = reinterpret_cast<int*>(s_scale + n);  // down items: expert, first member, count; total

  // The counter is read before this CTA adds anything (grid_bar_target);
  // TMEM is allocated while the ids load.
  auto init = [&]() {
    if (warp == 1) {
      tmem_alloc(&tmem_slot, FFN_TC_TMEM_COLS);
      tmem_relinquish();
      tc_fence_before();
    }
    if (threadIdx.x == 0) sync0 = ld_relaxed_gpu_u64(fa.sync);
  };
  route_build<true, decltype(init), kRoute>(r, fa.ids, n, fa.E, fa.K, true, MAX_SLOTS,
                                            fa.gu.status, init, fa.scale, s_scale);
  // Down items: every group's members in runs of at most DTC_N, in group
  // order (the order the two-kernel path's routing gives them).
  if (warp == 0) {
    const int nsg = *r.nsg;
    int total = 0;
    for (int g0 = 0; g0 < nsg; g0 += 32) {
      const int g = g0 + lane;
      const int cnt = g < nsg ? r.sg_cnt[g] : 0;
      const int ns = (cnt + DTC_N - 1) / DTC_N;
      int inc = ns;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      const int pos = total + inc - ns;
      for (int j = 0; j < ns; ++j) {
        dsg[pos + j] = r.sg_exp[g];
        dsg[n + pos + j] = r.sg_beg[g] + j * DTC_N;
        dsg[2 * n + pos + j] = min(DTC_N, cnt - j * DTC_N);
      }
      total += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) dsg[3 * n] = total;
  }
  __syncthreads();
  tc_fence_after();
  FusedCtx fx{base + fa.route_bytes, &r, s_scale, tmem_slot, fa.sync, 0ull};

  gate_up_tc_body<false, kRoute, true>(tm_gw, tm_x, nullptr, fa.gu, &fx);  // ends with __syncthreads

  // This CTA's h rows are stored (the barrier above): its share of the grid
  // barrier (release).  Every CTA gets here, also after a timed-out wait.
  if (threadIdx.x == 0) red_release_gpu_add_u64(fa.sync, grid_bar_share());
  RouteSmem rd = r;
  rd.sg_exp = dsg;
  rd.sg_beg = dsg + n;
  rd.sg_cnt = dsg + 2 * n;
  rd.nsg = dsg + 3 * n;
  fx.r = &rd;
  fx.target = grid_bar_target(sync0);
  down_tc_body<kTP, false, kRoute, true>(tm_dw, fa.dn, &fx);

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_slot, FFN_TC_TMEM_COLS);
  }
}

}  // namespace wdb
