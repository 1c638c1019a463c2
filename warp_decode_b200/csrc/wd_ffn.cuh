// The whole MoE FFN of a small decode batch in ONE launch, sm_100a:
//   h = silu(x . Wg) * (x . Wu)      (moe_gate_up_3d_batched_kernel,
//                                      csrc/moe_gate_up_3d_batched.cu:49-115)
//   y = sum_s scale_s * (h_s . Wd)   (moe_down_3d_batched_kernel,
//                                      csrc/moe_down_3d_batched.cu:45-122)
// The reference runs these as two launches with h in HBM between them; at
// decode batch sizes each launch costs several microseconds of ramp-up and
// tail next to a few microseconds of weight streaming, and the down weights
// cannot start streaming before gate_up has finished.
//
// Design (B200):
//  * Cooperative persistent grid, one CTA per SM (all CTAs co-resident):
//    8 consumer warps + 1 producer warp, the warp roles of the two SIMT
//    kernels.  Each consumer warp has its own ring; lane w of the producer
//    warp streams warp w's stage sequence into it with cp.async.bulk:
//    first its gate_up stages (items (group, neuron), gate and up row chunks),
//    then its down stages (items (group, chunk of this CTA's output rows)).
//    The producer never waits for h: down weights stream into the ring as soon
//    as gate_up stages free it, so HBM sees one continuous weight stream.
//  * Phase 1 (gate_up) writes h to global memory (L2-resident, 3 KB/token).
//  * Grid barrier (one thread per CTA, bounded wait, sense-reversing counter
//    in the caller's `sync` words): every CTA's h rows are visible before any
//    CTA reads h.  Then every CTA copies the call's h into shared memory (over
//    the x tile, no longer needed) with L2 loads.
//  * Phase 2 (down) is the SIMT down kernel's consumer: CTA c owns output rows
//    [c*H/G, (c+1)*H/G) for every token, per-warp FP32 tiles summed in a
//    fixed order: deterministic, no atomics on y.
#pragma once

#include "wd_down.cuh"

namespace wdb {

struct FfnArgs {
  const __nv_bfloat16* x;  // [B, H]
  const uint8_t* wgu;      // [E, 2I, H] bf16
  const uint8_t* wdn;      // [E, H, I] bf16
  const int32_t* ids;      // [B, K]
  const float* scale;      // [B, K]
  __nv_bfloat16* h;        // [B*K, I]: written in phase 1, read in phase 2
  uint32_t* sync;          // [0] arrivals, [1] generation (grid barrier)
  void* out;               // [B, H] bf16 or fp32
  int out_fp32;
  uint32_t* status;
  int B, E, K, H, I;
  int dedup;
  int depth;        // ring slots per consumer warp
  int stage_bytes;  // bytes per ring slot (multiple of 128)
  int kc;           // gate_up: weight elements per row chunk
  int rc;           // down: weight rows per chunk
  int lpr;          // down: lanes per weight row (8, 16 or 32)
  int rows_max;     // down: max output rows per CTA (ceil(H / gridDim.x))
  int xh_bytes;     // bytes of the shared x (phase 1) / h (phase 2) region
};

constexpr int FFN_THREADS = (NWARPS + 1) * 32;
constexpr int FFN_SYNC_WORDS = 2;
constexpr int FFN_MAX_SLOTS = 64;  // B * topk of one single-launch call

// Grid-barrier words used when the caller passes none (one pair per device,
// zero at module load).
__device__ __align__(8) uint32_t g_wd_ffn_sync[FFN_SYNC_WORDS] = {0u, 0u};

__host__ inline int ffn_smem_bytes(int depth, int stage_bytes, int xh_bytes, int B, int rows_max,
                                   int n, int E, bool dedup) {
  return NWARPS * depth * stage_bytes + ((xh_bytes + 127) / 128) * 128 +
         ((NWARPS * B * rows_max * 4 + 127) / 128) * 128 + ((n * 4 + 127) / 128) * 128 +
         (2 * NWARPS * depth + 1) * 8 + CTRL_INTS * 4 + route_smem_bytes(n, E, dedup);
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 16-byte load through L2 only (data written by other CTAs of this grid).
__device__ __forceinline__ uint4 ldcg16(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Grid-wide barrier for a co-resident grid, called by ONE thread per CTA
// after a CTA-wide barrier that orders the CTA's global writes before it.
// sync[0] counts arrivals and is reset to 0 by the last one, which then bumps
// the generation sync[1]; the others wait (bounded) for the bump.  The words
// are left as found apart from the generation, so the next launch on the same
// stream reuses them.  Returns false if the wait gave up.
__device__ inline bool grid_barrier(uint32_t* sync, uint32_t nctas) {
  const uint32_t gen0 = ld_acquire_gpu(sync + 1);  // before arriving
  __threadfence();                                 // this CTA's writes, gpu scope
  const uint32_t old = atomicAdd(sync, 1u);
  if (old == nctas - 1) {
    atomicExch(sync, 0u);
    __threadfence();
    st_release_gpu(sync + 1, gen0 + 1u);
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(sync + 1) == gen0) {
    if (globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) return false;
    __nanosleep(64);
  }
  __threadfence();
  return true;
}

__global__ void __launch_bounds__(FFN_THREADS, 1) moe_ffn_kernel(const FfnArgs a) {
  constexpr int NCW = NWARPS;
  constexpr int WB = 2;  // bf16 weights
  extern __shared__ __align__(128) uint8_t smem[];
  const int depth = a.depth;
  const int SB = a.stage_bytes;
  const int nslots = NCW * depth;
  const int n = a.B * a.K;
  const int I = a.I;
  const size_t H = (size_t)a.H;
  const uint32_t x_bytes = (uint32_t)((size_t)a.B * H * 2);
  const uint32_t h_bytes = (uint32_t)((size_t)n * I * 2);
  const int tile = a.B * a.rows_max;  // floats per warp tile
  uint8_t* p = smem;
  uint8_t* ring = p;
  p += (size_t)nslots * SB;
  uint8_t* xh = p;  // x in phase 1, h in phase 2
  p += ((a.xh_bytes + 127) / 128) * 128;
  float* tiles = reinterpret_cast<float*>(p);
  p += ((NCW * tile * 4 + 127) / 128) * 128;
  float* s_scale = reinterpret_cast<float*>(p);
  p += ((n * 4 + 127) / 128) * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(p);
  uint64_t* empty = full + nslots;
  uint64_t* xbar = empty + nslots;
  // ctrl: [0] abort, [8+w] stages issued for warp w, [16+w] stages consumed.
  volatile int* ctrl = reinterpret_cast<int*>(xbar + 1);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;

  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = (int)gridDim.x;

  if (threadIdx.x < nslots) {
    mbar_init(&full[threadIdx.x], 1);
    mbar_init(&empty[threadIdx.x], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 32 * NCW) {
    mbar_init(xbar, 1);
    ctrl[0] = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(xbar, x_bytes);
    bulk_g2s_big(xh, a.x, x_bytes, xbar, l2_policy_evict_last());
  }
  for (int i = threadIdx.x; i < NCW * tile; i += blockDim.x) tiles[i] = 0.f;
  route_build<true>(r, a.ids, n, a.E, a.K, dedup, GROUP_MAX, a.status, NoInit(), a.scale,
                    s_scale);  // ends with __syncthreads

  const int nsg = *r.nsg;
  // Phase 1 work: (group, neuron) items round-robin over CTAs, then warps.
  const int items1 = nsg * I;
  const int KC = a.kc;
  const int nchunks = (a.H + KC - 1) / KC;
  const int cta_items1 =
      items1 > (int)blockIdx.x ? (items1 - (int)blockIdx.x + G - 1) / G : 0;
  // Phase 2 work: (group, chunk of this CTA's rows) items round-robin over warps.
  const int r0 = (int)((long long)blockIdx.x * a.H / G);
  const int r1 = (int)((long long)(blockIdx.x + 1) * a.H / G);
  const int nrows = r1 - r0;
  const int RC = a.rc;
  const int cpg = (nrows + RC - 1) / RC;
  const int items2 = nsg * cpg;
  const size_t row_bytes = (size_t)I * WB;
  auto tot1 = [&](int w) {
    const int wi = cta_items1 > w ? (cta_items1 - w + NCW - 1) / NCW : 0;
    return wi * nchunks;
  };
  auto tot2 = [&](int w) { return items2 > w ? (items2 - w + NCW - 1) / NCW : 0; };
  auto stage1 = [&](int w, int s, int& c, int& sg, int& nn) {
    const int il = s / nchunks;
    c = s - il * nchunks;
    const int t = (int)blockIdx.x + (w + il * NCW) * G;
    sg = t / I;
    nn = t - sg * I;
  };
  auto stage2 = [&](int w, int s, int& g, int& ch) {
    const int j = w + s * NCW;
    g = j / cpg;
    ch = j - g * cpg;
  };

  if (warp == NCW) {
    // ------------- producer: lane w streams warp w's stages ---------------
    const int w = lane;
    const int t1 = w < NCW ? tot1(w) : 0;
    const int tot = w < NCW ? t1 + tot2(w) : 0;
    const uint64_t pol = l2_policy_evict_first();
    int iss = 0;
    uint64_t t_idle = globaltimer_ns();
    while (__any_sync(0xffffffffu, iss < tot)) {
      bool progress = false;
      if (iss < tot) {
        const int slot = w * depth + iss % depth;
        if (mbar_test(&empty[slot], ((uint32_t)(iss / depth) & 1u) ^ 1u)) {
          uint8_t* st = ring + (size_t)slot * SB;
          if (iss < t1) {
            int c, sg, nn;
            stage1(w, iss, c, sg, nn);
            const int e = max(r.sg_exp[sg], 0);  // invalid-id group: any valid rows
            const int kc = c * KC;
            const int klen = min(KC, a.H - kc);
            const size_t row_g = (size_t)e * 2 * I + nn;
            const uint32_t wbytes = (uint32_t)klen * WB;
            mbar_arrive_expect_tx(&full[slot], 2 * wbytes);
            bulk_g2s(st, a.wgu + (row_g * H + kc) * WB, wbytes, &full[slot], pol);
            bulk_g2s(st + (size_t)KC * WB, a.wgu + ((row_g + I) * H + kc) * WB, wbytes,
                     &full[slot], pol);
          } else {
            int g, ch;
            stage2(w, iss - t1, g, ch);
            const int nr = min(RC, nrows - ch * RC);
            const int e = max(r.sg_exp[g], 0);
            const size_t row0 = (size_t)e * H + r0 + ch * RC;
            const uint32_t tx = (uint32_t)(nr * row_bytes);
            mbar_arrive_expect_tx(&full[slot], tx);
            bulk_g2s(st, a.wdn + row0 * row_bytes, tx, &full[slot], pol);
          }
          ++iss;
          progress = true;
        }
      }
      if (__any_sync(0xffffffffu, progress)) {
        t_idle = globaltimer_ns();
      } else {
        if (__any_sync(0xffffffffu, ctrl[0] != 0)) break;
        __nanosleep(32);
        bool timeout = globaltimer_ns() - t_idle > WD_WAIT_LIMIT_NS;
        timeout = __shfl_sync(0xffffffffu, timeout, 0);
        if (timeout) {
          if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
          ctrl[0] = 1;
          break;
        }
      }
    }
    if (w < NCW) ctrl[8 + w] = iss;
  } else {
    // ------------------------------ consumers ------------------------------
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(xh);
    int pos = 0;  // ring position of the next stage
    if (!mbar_wait(xbar, 0)) {
      if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
    // ---- phase 1: gate_up + silu*up -> h (global) ----
    {
      const int total = tot1(warp);
      float ag[GROUP_MAX], ag2[GROUP_MAX], au[GROUP_MAX], au2[GROUP_MAX];
      const __nv_bfloat16* xrow[GROUP_MAX];
      int cnt = 0, beg = 0, e = 0;
      for (; pos < total; ++pos) {
        int c, sg, nn;
        stage1(warp, pos, c, sg, nn);
        if (c == 0) {
          e = r.sg_exp[sg];
          cnt = r.sg_cnt[sg];
          beg = r.sg_beg[sg];
#pragma unroll
          for (int m = 0; m < GROUP_MAX; ++m) {
            xrow[m] = xs + (size_t)r.mtok[beg + (m < cnt ? m : 0)] * H;
            ag[m] = 0.f;
            ag2[m] = 0.f;
            au[m] = 0.f;
            au2[m] = 0.f;
          }
        }
        const int slot = warp * depth + pos % depth;
        if (ctrl[0] || !mbar_wait(&full[slot], (uint32_t)(pos / depth) & 1u)) {
          if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
          ctrl[0] = 1;
          break;
        }
        if (e >= 0) {
          const uint8_t* st = ring + (size_t)slot * SB;
          const int kc = c * KC;
          const int klen = min(KC, a.H - kc);
          const __nv_bfloat16* xr[GROUP_MAX];
#pragma unroll
          for (int m = 0; m < GROUP_MAX; ++m) xr[m] = xrow[m] + kc;
          const uint8_t* gs = st;
          const uint8_t* us = st + (size_t)KC * WB;
          if (cnt == 1)
            gu_chunk<W_BF16, 1>(gs, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                                au2);
          else if (cnt == 2)
            gu_chunk<W_BF16, 2>(gs, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                                au2);
          else if (cnt <= 4)
            gu_chunk<W_BF16, 4>(gs, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                                au2);
          else
            gu_chunk<W_BF16, GROUP_MAX>(gs, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag,
                                        ag2, au, au2);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // slot back to the producer
        if (c == nchunks - 1) {
#pragma unroll
          for (int m = 0; m < GROUP_MAX; ++m) {
            if (m < cnt) {
              const float g = warp_sum(ag[m] + ag2[m]);
              const float u = warp_sum(au[m] + au2[m]);
              if (lane == m) {
                // A slot with an out-of-range expert id yields zeros.
                a.h[(size_t)r.members[beg + m] * I + nn] =
                    __float2bfloat16_rn(e >= 0 ? silu_f32(g) * u : 0.f);
              }
            }
          }
        }
      }
    }
    // ---- grid barrier: every CTA's h rows written before any is read ----
    named_barrier_sync(1, NCW * 32);
    if (threadIdx.x == 0 && !grid_barrier(a.sync, (uint32_t)G)) {
      raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
    named_barrier_sync(1, NCW * 32);
    // h of the whole call -> shared memory (over the x tile), through L2.
    __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(xh);
    if (!ctrl[0]) {
      const uint4* src = reinterpret_cast<const uint4*>(a.h);
      uint4* dst = reinterpret_cast<uint4*>(hs);
      for (int i = threadIdx.x; i < (int)(h_bytes / 16); i += NCW * 32) dst[i] = ldcg16(src + i);
    }
    named_barrier_sync(1, NCW * 32);
    // ---- phase 2: down + top-k weighted sum -> per-warp FP32 tiles ----
    if (!ctrl[0]) {
      const int t1 = tot1(warp);
      const int total = tot2(warp);
      const int lpr = a.lpr;
      const int rpp = 32 / lpr;  // rows per pass of the warp
      const int prow = lane / lpr;
      const int lj = lane - prow * lpr;
      const int nvec = I / 8;
      float* my_tile = tiles + (size_t)warp * tile;
      for (int s = 0; s < total; ++s, ++pos) {
        int g, ch;
        stage2(warp, s, g, ch);
        const int lr0 = ch * RC;
        const int nr = min(RC, nrows - lr0);
        const int e = r.sg_exp[g];
        const int cnt = r.sg_cnt[g];
        const int beg = r.sg_beg[g];
        const int slot = warp * depth + (t1 + s) % depth;
        if (ctrl[0] || !mbar_wait(&full[slot], (uint32_t)((t1 + s) / depth) & 1u)) {
          if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
          ctrl[0] = 1;
          break;
        }
        if (e >= 0) {  // a slot with an out-of-range expert id contributes nothing
          const uint8_t* st = ring + (size_t)slot * SB;
          if (cnt == 1)
            dn_item<W_BF16, 1>(st, nullptr, row_bytes, 0, nr, nvec, lpr, rpp, prow, lj, r, beg,
                               cnt, hs, true, I, s_scale, my_tile, a.rows_max, lr0);
          else if (cnt == 2)
            dn_item<W_BF16, 2>(st, nullptr, row_bytes, 0, nr, nvec, lpr, rpp, prow, lj, r, beg,
                               cnt, hs, true, I, s_scale, my_tile, a.rows_max, lr0);
          else if (cnt <= 4)
            dn_item<W_BF16, 4>(st, nullptr, row_bytes, 0, nr, nvec, lpr, rpp, prow, lj, r, beg,
                               cnt, hs, true, I, s_scale, my_tile, a.rows_max, lr0);
          else
            dn_item<W_BF16, GROUP_MAX>(st, nullptr, row_bytes, 0, nr, nvec, lpr, rpp, prow, lj,
                                       r, beg, cnt, hs, true, I, s_scale, my_tile, a.rows_max,
                                       lr0);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }
    if (lane == 0) ctrl[16 + warp] = pos;
  }
  __syncthreads();
  if (ctrl[0]) {
    // A wait gave up: let issued but unconsumed copies land, then leave
    // without writing y (the status word says so).
    if (warp < NCW && lane == 0)
      for (int q = ctrl[16 + warp]; q < ctrl[8 + warp]; ++q)
        if (!mbar_wait(&full[warp * depth + q % depth], (uint32_t)(q / depth) & 1u)) break;
    return;
  }
  // y = sum of the 8 warp tiles in a fixed order.
  for (int i = threadIdx.x; i < a.B * nrows; i += blockDim.x) {
    const int b = i / nrows;
    const int lr = i - b * nrows;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) v += tiles[(size_t)w * tile + b * a.rows_max + lr];
    const size_t o = (size_t)b * H + r0 + lr;
    if (a.out_fp32)
      reinterpret_cast<float*>(a.out)[o] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(v);
  }
}

}  // namespace wdb
