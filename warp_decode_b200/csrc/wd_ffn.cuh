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
//  * Cooperative persistent grid, one CTA per SM (all CTAs co-resident),
//    up to FFN_MAX_WARPS warps (the launch's block size; the host takes the
//    most that fit next to a two-slot ring per warp: more warps spread the
//    CTA's gate_up items and down chunks thinner, so the busiest warp's
//    share of the weight stream, not the CTA's, sets the phase times).
//    Every warp owns a ring of `depth` shared-memory slots and
//    feeds it itself: after consuming stage s it issues stage s + depth with
//    cp.async.bulk (no producer warp to wake, no empty barriers).  A warp's
//    stage sequence is its gate_up stages (items (group, neuron): gate and up
//    row chunks) followed by its down stages (items (group, chunk of this
//    CTA's output rows)), so down weights stream into the ring while gate_up
//    still computes and HBM sees one continuous weight stream.
//  * Phase 1 (gate_up) writes h to global memory (L2-resident, 3 KB/token).
//  * Grid barrier (one thread per CTA, bounded wait): a 64-bit arrival
//    counter in the caller's `sync` words that only ever grows (every launch
//    adds exactly GRID_BAR_UNITS, grid_bar_share), so the target is known from
//    the value read at kernel entry and arrival is a single release reduction.  Then
//    every CTA copies the call's h into shared memory (over the x tile, no
//    longer needed) with L2 loads.
//  * Phase 2 (down): CTA c owns output rows [c*H/G, (c+1)*H/G) for every
//    token; per-warp FP32 tiles summed in a fixed order (deterministic, no
//    atomics on y).
//  * Tensor parallelism (kTP): the CTA's FP32 rows are this rank's partial
//    sums; they are all-reduced over NVLink peer stores of 8-byte (value,
//    epoch) packets, one-shot or two-shot (the exchange of the tcgen05 down
//    kernel, TpArgs / TpCall): y is the all-reduced bf16 output, identical
//    bits on every rank, with no other launch.
//  * Short code on the launch's critical path: after an L2 flush the kernel's
//    instructions come from DRAM, and each taken branch into code not yet
//    fetched costs about a DRAM latency.  Routing compiles only the
//    <= 64-slot path, gate_up has two accumulate variants (1 member / up to
//    8), and down is one compact loop nest.
#pragma once

#include "wd_down.cuh"
#include "wd_down_tc.cuh"
#include "wd_tc.cuh"

namespace wdb {

struct FfnArgs {
  const __nv_bfloat16* x;  // [B, H]
  const uint8_t* wgu;      // [E, 2I, H] bf16
  const uint8_t* wdn;      // [E, H, I] bf16
  const int32_t* ids;      // [B, K]
  const float* scale;      // [B, K]
  __nv_bfloat16* h;        // [B*K, I]: written in phase 1, read in phase 2
  unsigned long long* sync;  // grid-barrier arrival counter (8 bytes)
  void* out;               // [B, H] bf16 or fp32
  int out_fp32;
  uint32_t* status;
  int B, E, K, H, I;
  int dedup;
  int depth;        // ring slots per warp
  int stage_bytes;  // bytes per ring slot (multiple of 128)
  int kc;           // gate_up: weight elements per row chunk
  int rc;           // down: weight rows per chunk
  int rows_max;     // down: max output rows per CTA (ceil(H / gridDim.x))
  int xh_bytes;     // bytes of the shared x (phase 1) / h (phase 2) region
  TpArgs tp;        // fused all-reduce (kTP): y = bf16 sum over the group's ranks
};

// Warps of one CTA: at most FFN_MAX_WARPS (launch bounds), chosen per call.
// Measured on B200 (H 4096, I 192, E 128, top-8, cold, us, 8 -> 11 warps):
// B = 1 22.7 -> 20.5, B = 2 30.8 -> 26.6, B = 4 43.1 -> 40.0; 12 warps no
// better at B = 1, 2 and too large for B = 4; 6 warps slower.
constexpr int FFN_MAX_WARPS = 11;
constexpr int FFN_THREADS = FFN_MAX_WARPS * 32;
// ctrl words: [0] abort flag, [FFN_CTRL_ISSUED + w] stages issued by warp w,
// [FFN_CTRL_POS + w] stages it consumed (read back after an abort).
constexpr int FFN_CTRL_ISSUED = 4;
constexpr int FFN_CTRL_POS = FFN_CTRL_ISSUED + FFN_MAX_WARPS;
static_assert(FFN_CTRL_POS + FFN_MAX_WARPS <= CTRL_INTS, "ctrl words");
constexpr int FFN_MAX_SLOTS = 64;  // B * topk of one single-launch call

// Grid-barrier counter used when the caller passes none (one per device,
// zero at module load).
__device__ unsigned long long g_wd_ffn_sync = 0ull;

__host__ inline int ffn_smem_bytes(int nw, int depth, int stage_bytes, int xh_bytes, int B,
                                   int rows_max, int n, int E, bool dedup) {
  return nw * depth * stage_bytes + ((xh_bytes + 127) / 128) * 128 +
         ((nw * B * rows_max * 4 + 127) / 128) * 128 + ((n * 4 + 127) / 128) * 128 +
         (nw * depth + 1) * 8 + CTRL_INTS * 4 + route_smem_bytes(n, E, dedup);
}

// Generic-proxy reads of a shared-memory slot before an async-proxy (bulk
// copy) write into it.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One down stage: nr (<= 16 per pass) weight rows of one expert in shared
// memory against the group's cnt members' h rows (shared memory).  Two lanes
// per row (16 rows per pass), each summing every other 16-byte vector of the
// row; lane pairs start at a row-dependent vector (rotation by 2 * row), so
// the 8 lanes of a shared-memory phase hit 8 different bank groups even when
// the row pitch is a multiple of 128 bytes (measured: 1.5x faster with 8
// warps than without the rotation).  Four vectors in flight per lane.
// scale * dot goes into the warp's own tile.  Every loop that contains a
// shuffle has a warp-uniform trip count.
__device__ __forceinline__ void ffn_down_stage(const uint8_t* st, int row_bytes, int nr, int nvec,
                                               int lane, const RouteSmem& r, int beg, int cnt,
                                               const __nv_bfloat16* hs, int I,
                                               const float* s_scale, float* my_tile,
                                               int rows_max, int lr0) {
  const int prow = lane >> 1, q = lane & 1;
#pragma unroll 1
  for (int rb = 0; rb < nr; rb += 16) {
    const int row = rb + prow;
    const bool live = row < nr;
    const uint8_t* wrow = st + (size_t)(live ? row : 0) * row_bytes;
    // first vector: rotated by 2 * row when nvec is even (the rotation then
    // keeps each lane on its own parity class of vectors)
    const int v0 = (nvec & 1) ? q : (2 * row + q) % nvec;
#pragma unroll 1
    for (int m = 0; m < cnt; ++m) {
      const int slot_i = r.members[beg + m];
      const __nv_bfloat16* hr = hs + (size_t)slot_i * I;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (live) {
        int v = v0;  // == it when nvec is odd (no wrap)
        int it = q;  // vectors q, q + 2, ... of the row, rotated
        for (; it + 6 < nvec; it += 8) {
          int va = v, vb = va + 2, vc = va + 4, vd = va + 6;
          vb -= vb >= nvec ? nvec : 0;
          vc -= vc >= nvec ? nvec : 0;
          vd -= vd >= nvec ? nvec : 0;
          const uint4 wa = lds16(wrow + va * 16), wb = lds16(wrow + vb * 16);
          const uint4 wc = lds16(wrow + vc * 16), wd = lds16(wrow + vd * 16);
          const uint4 ha = lds16(hr + va * 8), hb = lds16(hr + vb * 8);
          const uint4 hc = lds16(hr + vc * 8), hd = lds16(hr + vd * 8);
          dot8_bf16(a0, a1, ha, wa);
          dot8_bf16(a2, a3, hb, wb);
          dot8_bf16(a0, a1, hc, wc);
          dot8_bf16(a2, a3, hd, wd);
          v = vd + 2;
          v -= v >= nvec ? nvec : 0;
        }
        for (; it < nvec; it += 2) {
          dot8_bf16(a0, a1, lds16(hr + v * 8), lds16(wrow + v * 16));
          v += 2;
          v -= v >= nvec ? nvec : 0;
        }
      }
      float acc = (a0 + a1) + (a2 + a3);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (live && q == 0) {
        float* dst = &my_tile[r.mtok[beg + m] * rows_max + lr0 + row];
        *dst = fmaf(s_scale[slot_i], acc, *dst);
      }
    }
  }
}

template <bool kTP>
__global__ void __launch_bounds__(FFN_THREADS, 1) moe_ffn_kernel(const FfnArgs a) {
  const int NCW = (int)(blockDim.x >> 5);  // warps of this launch (<= FFN_MAX_WARPS)
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
  uint64_t* xbar = full + nslots;
  // ctrl: [0] abort, [FFN_CTRL_ISSUED + w] stages issued by warp w,
  // [FFN_CTRL_POS + w] stages consumed.
  volatile int* ctrl = reinterpret_cast<int*>(xbar + 1);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;

  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = (int)gridDim.x;
  const uint32_t tp_ep = kTP ? a.tp.epochs[blockIdx.x] + 1u : 0u;  // this call's epoch

  // Barrier counter at entry (used at the barrier): every earlier launch
  // added exactly GRID_BAR_UNITS and this CTA has not arrived yet, so
  // floor(count / GRID_BAR_UNITS) counts the earlier launches.
  unsigned long long sync0 = 0ull;
  if (threadIdx.x == 0) {
    mbar_init(xbar, 1);
    ctrl[0] = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(xbar, x_bytes);
    bulk_g2s_big(xh, a.x, x_bytes, xbar, l2_policy_evict_last());
    sync0 = ld_relaxed_gpu_u64(a.sync);
  }
  if (threadIdx.x < nslots) {
    mbar_init(&full[threadIdx.x], 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < NCW * tile; i += blockDim.x) tiles[i] = 0.f;
  route_build<true, NoInit, ROUTE_SMALL>(r, a.ids, n, a.E, a.K, dedup, GROUP_MAX, a.status, NoInit(),
                                  a.scale, s_scale);  // ends with __syncthreads

  const int nsg = *r.nsg;
  // Phase 1 work: (group, neuron) items round-robin over CTAs, then warps.
  const int items1 = nsg * I;
  const int KC = a.kc;
  const int nchunks = (a.H + KC - 1) / KC;
  const int cta_items1 =
      items1 > (int)blockIdx.x ? (items1 - (int)blockIdx.x + G - 1) / G : 0;
  const int t1 = (cta_items1 > warp ? (cta_items1 - warp + NCW - 1) / NCW : 0) * nchunks;
  // Phase 2 work: (group, chunk of this CTA's rows) items round-robin over warps.
  const int r0 = (int)((long long)blockIdx.x * a.H / G);
  const int r1 = (int)((long long)(blockIdx.x + 1) * a.H / G);
  const int nrows = r1 - r0;
  const int RC = a.rc;
  const int cpg = (nrows + RC - 1) / RC;
  const int items2 = nsg * cpg;
  const int t2 = items2 > warp ? (items2 - warp + NCW - 1) / NCW : 0;
  const int total = t1 + t2;
  const int row_bytes = I * WB;
  const uint64_t pol = l2_policy_evict_first();
  uint8_t* my_ring = ring + (size_t)warp * depth * SB;
  uint64_t* my_full = full + warp * depth;

  // Stage s of this warp: phase 1 -> item il = s / nchunks, chunk c; phase 2
  // -> item j = warp + (s - t1) * NCW.
  auto stage1 = [&](int s, int& c, int& sg, int& nn) {
    const int il = s / nchunks;
    c = s - il * nchunks;
    const int t = (int)blockIdx.x + (warp + il * NCW) * G;
    sg = t / I;
    nn = t - sg * I;
  };
  auto stage2 = [&](int s, int& g, int& ch) {
    const int j = warp + (s - t1) * NCW;
    g = j / cpg;
    ch = j - g * cpg;
  };
  // Lane 0 issues stage s into slot s % depth (whose previous stage has been
  // consumed by this warp).
  auto issue = [&](int s) {
    const int k = s % depth;
    uint8_t* st = my_ring + (size_t)k * SB;
    if (s < t1) {
      int c, sg, nn;
      stage1(s, c, sg, nn);
      const int e = max(r.sg_exp[sg], 0);  // invalid-id group: any valid rows
      const int kc = c * KC;
      const int klen = min(KC, a.H - kc);
      const size_t row_g = (size_t)e * 2 * I + nn;
      const uint32_t wbytes = (uint32_t)klen * WB;
      mbar_arrive_expect_tx(&my_full[k], 2 * wbytes);
      bulk_g2s(st, a.wgu + (row_g * H + kc) * WB, wbytes, &my_full[k], pol);
      bulk_g2s(st + (size_t)KC * WB, a.wgu + ((row_g + I) * H + kc) * WB, wbytes, &my_full[k],
               pol);
    } else {
      int g, ch;
      stage2(s, g, ch);
      const int nr = min(RC, nrows - ch * RC);
      const int e = max(r.sg_exp[g], 0);
      const size_t row0 = (size_t)e * H + r0 + ch * RC;
      const uint32_t tx = (uint32_t)nr * (uint32_t)row_bytes;
      mbar_arrive_expect_tx(&my_full[k], tx);
      bulk_g2s(st, a.wdn + row0 * row_bytes, tx, &my_full[k], pol);
    }
  };
  int issued = min(depth, total);
  if (lane == 0)
    for (int s = 0; s < issued; ++s) issue(s);

  const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(xh);
  int pos = 0;  // next stage to consume
  // Consume stage `pos`: every lane waits for it (bounded); the warp agrees
  // on the outcome, so all lanes leave a loop together.  false = give up.
  auto wait_stage = [&]() {
    bool ok = __all_sync(0xffffffffu, ctrl[0] == 0);
    if (ok) ok = mbar_wait(&my_full[pos % depth], (uint32_t)(pos / depth) & 1u);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) {
      raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
    return ok;
  };
  // Stage `pos` consumed: refill its slot with stage pos + depth.
  auto release_stage = [&]() {
    __syncwarp();
    if (issued < total) {
      if (lane == 0) {
        fence_proxy_async_shared();
        issue(issued);
      }
      ++issued;
    }
    ++pos;
  };

  if (!mbar_wait(xbar, 0)) {
    if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
    ctrl[0] = 1;
  }
  // ---- phase 1: gate_up + silu*up -> h (global) ----
  {
    float ag[GROUP_MAX], ag2[GROUP_MAX], au[GROUP_MAX], au2[GROUP_MAX];
    const __nv_bfloat16* xrow[GROUP_MAX];
    int cnt = 0, beg = 0, e = 0;
    while (pos < t1) {
      int c, sg, nn;
      stage1(pos, c, sg, nn);
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
      if (!wait_stage()) break;
      if (e >= 0) {
        const uint8_t* st = my_ring + (size_t)(pos % depth) * SB;
        const int kc = c * KC;
        const int klen = min(KC, a.H - kc);
        const __nv_bfloat16* xr[GROUP_MAX];
#pragma unroll
        for (int m = 0; m < GROUP_MAX; ++m) xr[m] = xrow[m] + kc;
        const uint8_t* us = st + (size_t)KC * WB;
        if (cnt == 1)
          gu_chunk<W_BF16, 1>(st, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                              au2);
        else if (cnt == 2)
          gu_chunk<W_BF16, 2>(st, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                              au2);
        else if (cnt <= 4)
          gu_chunk<W_BF16, 4>(st, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag, ag2, au,
                              au2);
        else
          gu_chunk<W_BF16, GROUP_MAX>(st, us, nullptr, nullptr, klen, xr, true, cnt, lane, ag,
                                      ag2, au, au2);
      }
      release_stage();
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
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long bar_target = grid_bar_target(sync0);
    red_release_gpu_add_u64(a.sync, grid_bar_share());
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    while (ld_acquire_gpu_u64(a.sync) < bar_target) {
      if (globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) { ok = false; break; }
      __nanosleep(32);
    }
    if (!ok) {
      raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
  }
  __syncthreads();
  // h of the whole call -> shared memory (over the x tile), through L2.
  __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(xh);
  if (!ctrl[0]) {
    const uint4* src = reinterpret_cast<const uint4*>(a.h);
    uint4* dst = reinterpret_cast<uint4*>(hs);
    const int nv = (int)(h_bytes / 16);
    const int nt = (int)blockDim.x;
    for (int i = threadIdx.x; i < nv; i += 4 * nt) {
      uint4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i + q * nt < nv) v[q] = ldcg16(src + i + q * nt);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i + q * nt < nv) dst[i + q * nt] = v[q];
    }
  }
  __syncthreads();
  // ---- phase 2: down + top-k weighted sum -> per-warp FP32 tiles ----
  if (!ctrl[0]) {
    const int nvec = I / 8;
    float* my_tile = tiles + (size_t)warp * tile;
    while (pos < total) {
      int g, ch;
      stage2(pos, g, ch);
      const int lr0 = ch * RC;
      const int nr = min(RC, nrows - lr0);
      const int e = r.sg_exp[g];
      if (!wait_stage()) break;
      if (e >= 0)  // a slot with an out-of-range expert id contributes nothing
        ffn_down_stage(my_ring + (size_t)(pos % depth) * SB, row_bytes, nr, nvec, lane, r,
                       r.sg_beg[g], r.sg_cnt[g], hs, I, s_scale, my_tile, a.rows_max, lr0);
      release_stage();
    }
  }
  if (lane == 0) {
    ctrl[FFN_CTRL_ISSUED + warp] = issued;
    ctrl[FFN_CTRL_POS + warp] = pos;
  }
  __syncthreads();
  if (ctrl[0]) {
    // A wait gave up: let issued but unconsumed copies land, then leave
    // without writing y (the status word says so).  With the fused
    // all-reduce the call still counts (epochs stay in step with the peers,
    // which time out on this rank's missing packets).
    if (lane == 0)
      for (int q = ctrl[FFN_CTRL_POS + warp]; q < ctrl[FFN_CTRL_ISSUED + warp]; ++q)
        if (!mbar_wait(&my_full[q % depth], (uint32_t)(q / depth) & 1u)) break;
    if (kTP && threadIdx.x == 0)
      for (int c2 = (int)blockIdx.x; c2 < a.tp.max_ctas; c2 += G) a.tp.epochs[c2] = tp_ep;
    return;
  }
  if constexpr (kTP) {
    // This rank's partial rows go out first (TpCall: one-shot or two-shot);
    // then tp_collect: the rows this rank sums, in rank order, and (two-shot)
    // the rows whose owner sends the result.  A packet that does not arrive
    // within 2 s gives a zero row and raises WD_STATUS_WAIT_TIMEOUT.
    const TpCall xc{a.tp, tp_ep, a.H};
    for (int i = threadIdx.x; i < a.B * nrows; i += blockDim.x) {
      const int b = i / nrows;
      const int lr = i - b * nrows;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) v += tiles[(size_t)w * tile + b * a.rows_max + lr];
      xc.push(b, r0 + lr, v);
    }
    tp_collect(xc, a.B * nrows, [&](int i, int& b, int& row) {
      b = i / nrows;
      row = r0 + (i - b * nrows);
      return true;
    }, reinterpret_cast<__nv_bfloat16*>(a.out), a.status);
    if (threadIdx.x == 0)
      for (int c2 = (int)blockIdx.x; c2 < a.tp.max_ctas; c2 += G) a.tp.epochs[c2] = tp_ep;
  } else {
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
}

}  // namespace wdb
