// down projection + top-k weighted sum for MoE decode, sm_100a.
//
// Computes y[b, j] = sum_s topk_scale[b,s] * (h[b*topk+s, :] . Wd[e_s, j, :])
// (the operation of moe_down_3d_batched_kernel,
//  csrc/moe_down_3d_batched.cu:45-122 of the reference), with FP32 products
// and FP32 accumulation (the reference rounds each product to bf16 first).
//
// Design (B200):
//  * Persistent grid, one CTA per SM: 8 consumer warps + 1 producer warp.
//    CTA c owns output rows [c*H/G, (c+1)*H/G) for every token, so the top-k
//    reduction never leaves the CTA: no atomics, no scratch memory.
//  * Work items are (routing group, chunk of the CTA's rows): a group is up
//    to GROUP_MAX slots sharing an expert (each expert's rows are read from
//    HBM once per call) and a chunk is >= 4 KB of contiguous weight rows, the
//    size below which bulk copies stop saturating HBM on B200.  Items go to
//    consumer warps round-robin; lane w of the producer warp streams consumer
//    warp w's items with cp.async.bulk into ring slots only that warp uses.
//  * h of the whole call and the top-k scales sit in shared memory.  `lpr`
//    lanes share a weight row (16-byte vectors), dot it with each member's h
//    row (bf16 inputs, FP32 accumulation), reduce with shuffles and add
//    scale * dot into the warp's own FP32 tile [B][rows].  At the end the 8
//    tiles are summed in a fixed order: deterministic, one store per output.
//  * Programmatic dependent launch: routing and the first `depth` weight
//    stages of every warp are issued before griddepcontrol.wait, i.e. while a
//    preceding gate_up grid still streams.  h and topk_scale are read only
//    after the wait.  topk_ids are re-read after the wait; if they changed
//    (possible only if the preceding kernel wrote them after signalling
//    early), the prefetched stages are discarded and the routing rebuilt.
#pragma once

#include "wd_gate_up.cuh"

namespace wdb {

struct DownArgs {
  const __nv_bfloat16* h;   // [B*K, I]
  const uint8_t* w;         // [E, H, I] bf16 or e4m3
  const uint8_t* wscale;    // [E, H, I/32] ue8m0 (e4m3 only)
  const int32_t* ids;       // [B, K]
  const float* scale;       // [B, K]
  void* out;                // [B, H] bf16 or fp32
  int out_fp32;
  uint32_t* status;
  int B, E, K, H, I;
  int dedup;
  int depth;        // ring slots per consumer warp
  int rc;           // weight rows per chunk (item)
  int lpr;          // lanes per weight row: 8, 16 or 32
  int stage_bytes;  // bytes per ring slot (weights + scales), multiple of 128
  int rows_max;     // max rows per CTA (ceil(H / gridDim.x))
  int h_smem;       // 1: h staged in shared memory
};

constexpr int DN_THREADS = (NWARPS + 1) * 32;

template <int FMT>
__host__ __device__ inline int down_scale_area(int rc, int I) {
  return FMT == W_E4M3 ? ((rc * (I / 32) + 32 + 15) / 16) * 16 : 0;
}

__host__ inline int down_smem_bytes(int depth, int stage_bytes, int h_bytes, int B, int rows_max,
                                    int n, int E, bool dedup) {
  return NWARPS * depth * stage_bytes + ((h_bytes + 127) / 128) * 128 +
         ((NWARPS * B * rows_max * 4 + 127) / 128) * 128 + ((n * 4 + 127) / 128) * 128 +
         (2 * NWARPS * depth + 1) * 8 + CTRL_INTS * 4 + route_smem_bytes(n, E, dedup);
}

// acc[m] += row . h[member m] over this lane's vectors (v = lj, lj+lpr, ...).
template <int FMT, int MAXM>
__device__ __forceinline__ void dn_row(const uint8_t* __restrict__ wrow, const uint8_t* srow,
                                       int nvec, int lj, int lpr,
                                       const __nv_bfloat16* const (&hr)[GROUP_MAX], bool hsm,
                                       int cnt, float (&acc)[MAXM], float (&acc2)[MAXM]) {
  if constexpr (FMT == W_BF16) {
#pragma unroll 2
    for (int v = lj; v < nvec; v += lpr) {
      const uint4 wv = lds16(wrow + v * 16);
#pragma unroll
      for (int m = 0; m < MAXM; ++m)
        if (m < cnt) dot8_bf16(acc[m], acc2[m], act16(hr[m] + v * 8, hsm), wv);
    }
  } else {
    // E4M3: decoded to exact bf16 patterns (scaled by 2^-120), the bf16 FMA,
    // then 2^120 x the block scale once per 16-element vector.
#pragma unroll 2
    for (int v = lj; v < nvec; v += lpr) {
      uint32_t wb[8];
      const bool nan_byte = e4m3x16_to_bf16(lds16(wrow + v * 16), wb);
      const uint32_t s = srow[v >> 1];
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < cnt) {
          float p = 0.f, p2 = 0.f;
          dot16_e4m3(p, p2, act16(hr[m] + v * 16, hsm), act16(hr[m] + v * 16 + 8, hsm), wb);
          acc[m] = mx_block_fma(p, s, nan_byte, acc[m]);
          acc2[m] = mx_block_fma(p2, s, nan_byte, acc2[m]);
        }
      }
    }
  }
}

// One staged item (nr rows of one expert) for the MAXM-bounded group members:
// per pass of rpp rows, lpr lanes per row; scale * dot goes into my_tile.
template <int FMT, int MAXM>
__device__ __forceinline__ void dn_item(const uint8_t* __restrict__ st, const uint8_t* sbase,
                                        size_t row_bytes, int sc_row, int nr, int nvec, int lpr,
                                        int rpp, int prow, int lj, const RouteSmem& r, int beg,
                                        int cnt, const __nv_bfloat16* hbase, bool hsm, int I,
                                        const float* __restrict__ s_scale, float* my_tile,
                                        int rows_max, int lr0) {
  const __nv_bfloat16* hr[GROUP_MAX];
  float sc[MAXM];
  int tok[MAXM];
#pragma unroll
  for (int m = 0; m < GROUP_MAX; ++m) hr[m] = hbase;
#pragma unroll
  for (int m = 0; m < MAXM; ++m) {
    const int at = beg + (m < cnt ? m : 0);
    const int slot_i = r.members[at];
    hr[m] = hbase + (size_t)slot_i * I;
    sc[m] = s_scale[slot_i];
    tok[m] = r.mtok[at];
  }
  // A lane's rows of the item are prow, prow + rpp, ...; up to DN_ROWS of
  // them are computed together so their load/FMA/shuffle chains overlap.
  constexpr int DN_ROWS = MAXM <= 2 ? 4 : (MAXM <= 4 ? 2 : 1);
  for (int rb = 0; rb < nr; rb += DN_ROWS * rpp) {
    float acc[DN_ROWS][MAXM], acc2[DN_ROWS][MAXM];
#pragma unroll
    for (int q = 0; q < DN_ROWS; ++q)
#pragma unroll
      for (int m = 0; m < MAXM; ++m) { acc[q][m] = 0.f; acc2[q][m] = 0.f; }
#pragma unroll
    for (int q = 0; q < DN_ROWS; ++q) {
      const int row = rb + q * rpp + prow;
      if (row < nr)
        dn_row<FMT, MAXM>(st + (size_t)row * row_bytes,
                          FMT == W_E4M3 ? sbase + (size_t)row * sc_row : nullptr, nvec, lj, lpr,
                          hr, hsm, cnt, acc[q], acc2[q]);
    }
#pragma unroll
    for (int q = 0; q < DN_ROWS; ++q)
#pragma unroll
      for (int m = 0; m < MAXM; ++m) acc[q][m] += acc2[q][m];
    for (int o = lpr >> 1; o > 0; o >>= 1) {
#pragma unroll
      for (int q = 0; q < DN_ROWS; ++q)
#pragma unroll
        for (int m = 0; m < MAXM; ++m)
          if (m < cnt) acc[q][m] += __shfl_xor_sync(0xffffffffu, acc[q][m], o);
    }
    if (lj == 0) {
#pragma unroll
      for (int q = 0; q < DN_ROWS; ++q) {
        const int row = rb + q * rpp + prow;
        if (row < nr) {
#pragma unroll
          for (int m = 0; m < MAXM; ++m) {
            if (m < cnt) {
              float* dst = &my_tile[tok[m] * rows_max + lr0 + row];
              *dst = fmaf(sc[m], acc[q][m], *dst);
            }
          }
        }
      }
    }
  }
}

// kRoute: routing code compiled for this launch's slot count (RouteMode).
template <int FMT, int kRoute>
__global__ void __maxnreg__(FMT == W_E4M3 ? 96 : 112) moe_down_kernel(const DownArgs a) {
  constexpr int WB = (FMT == W_BF16) ? 2 : 1;
  constexpr int EPV = (FMT == W_BF16) ? 8 : 16;
  constexpr int NCW = NWARPS;

  extern __shared__ __align__(128) uint8_t smem[];
  const int depth = a.depth;
  const int SB = a.stage_bytes;
  const int nslots = NCW * depth;
  const int n = a.B * a.K;
  const int I = a.I;
  const uint32_t h_bytes = (uint32_t)((size_t)n * I * 2);
  const int tile = a.B * a.rows_max;  // floats per warp tile
  uint8_t* p = smem;
  uint8_t* ring = p;
  p += (size_t)nslots * SB;
  __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(p);
  p += a.h_smem ? ((h_bytes + 127) / 128) * 128 : 0;
  float* tiles = reinterpret_cast<float*>(p);
  p += ((NCW * tile * 4 + 127) / 128) * 128;
  float* s_scale = reinterpret_cast<float*>(p);
  p += ((n * 4 + 127) / 128) * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(p);
  uint64_t* empty = full + nslots;
  uint64_t* hbar = empty + nslots;
  // ctrl: [0] abort, [1] routing changed, [8+w] issued, [16+w] consumed,
  // [24+w] prefetched before the routing check.
  volatile int* ctrl = reinterpret_cast<int*>(hbar + 1);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;

  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = (int)((long long)blockIdx.x * a.H / gridDim.x);
  const int r1 = (int)((long long)(blockIdx.x + 1) * a.H / gridDim.x);
  const int nrows = r1 - r0;
  const int RC = a.rc;
  const int cpg = (nrows + RC - 1) / RC;  // chunks per group in this CTA
  const size_t row_bytes = (size_t)I * WB;
  const int sc_off = RC * (int)row_bytes;

  if (threadIdx.x < nslots) {
    mbar_init(&full[threadIdx.x], 1);
    mbar_init(&empty[threadIdx.x], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 32 * NCW) {
    mbar_init(hbar, 1);
    ctrl[0] = 0;
    ctrl[1] = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < NCW * tile; i += blockDim.x) tiles[i] = 0.f;
  route_build<false, NoInit, kRoute>(r, a.ids, n, a.E, a.K, dedup, GROUP_MAX,
                                     a.status);  // before the wait: re-checked

  auto warp_total = [&](int w) {
    const int items = *r.nsg * cpg;
    return items > w ? (items - w + NCW - 1) / NCW : 0;
  };

  // Stage s of warp w = item j = w + s*NCW -> group j / cpg, row chunk j % cpg.
  int pre = 0;  // stages issued before the routing check (per warp, by lane w)
  if (warp == NCW && lane < NCW) {
    // ---- prefetch: weights only, before the dependency wait ----
    const int w = lane;
    pre = min(depth, warp_total(w));
    const uint64_t pol = l2_policy_evict_first();
    for (int s = 0; s < pre; ++s) {
      const int j = w + s * NCW;
      const int g = j / cpg;
      const int ch = j - g * cpg;
      const int nr = min(RC, nrows - ch * RC);
      const int e = max(r.sg_exp[g], 0);
      const int slot = w * depth + s;
      uint8_t* st = ring + (size_t)slot * SB;
      const size_t row0 = (size_t)e * a.H + r0 + ch * RC;
      uint32_t tx = (uint32_t)(nr * row_bytes);
      if constexpr (FMT == W_E4M3) {
        const uintptr_t s0 = (uintptr_t)(a.wscale + row0 * (I / 32));
        const uintptr_t s1 = s0 + (uintptr_t)nr * (I / 32);
        const uint8_t* s_src = (const uint8_t*)(s0 & ~(uintptr_t)15);
        const uint32_t s_len = (uint32_t)(((s1 + 15) & ~(uintptr_t)15) - (uintptr_t)s_src);
        mbar_arrive_expect_tx(&full[slot], tx + s_len);
        bulk_g2s(st + sc_off, s_src, s_len, &full[slot], pol);
      } else {
        mbar_arrive_expect_tx(&full[slot], tx);
      }
      bulk_g2s(st, a.w + row0 * row_bytes, tx, &full[slot], pol);
    }
    ctrl[8 + w] = pre;   // issued so far (the producer keeps this current)
    ctrl[24 + w] = pre;  // prefetched before the routing check (fixed)
  }

  // ---- dependency wait: h and topk_scale come from the preceding grid ----
  pdl_wait_primary();
  if (warp < NCW) {
    if (threadIdx.x == 0 && a.h_smem) {
      mbar_arrive_expect_tx(hbar, h_bytes);
      bulk_g2s_big(hs, a.h, h_bytes, hbar, l2_policy_evict_last());
    }
    bool changed = false;
    for (int i = threadIdx.x; i < n; i += NCW * 32) {
      s_scale[i] = __ldg(a.scale + i);
      int e = __ldg(a.ids + i);
      if (e < 0 || e >= a.E) e = -1;
      changed |= (e != r.ids[i]);
    }
    if (__any_sync(0xffffffffu, changed) && lane == 0) ctrl[1] = 1;
  }
  __syncthreads();
  const bool changed = ctrl[1] != 0;
  int pos0 = 0;  // ring position of the current routing's stage 0 (consumers)
  if (changed) {
    // The preceding kernel rewrote topk_ids after signalling early: rebuild
    // from the settled ids; prefetched stages are drained, not used.
    if (threadIdx.x == 0) raise_status(a.status, WD_STATUS_ROUTING_CHANGED);
    route_build<false, NoInit, kRoute>(r, a.ids, n, a.E, a.K, dedup, GROUP_MAX, a.status);
    if (warp < NCW) pos0 = ctrl[24 + warp];
  }

  if (warp == NCW) {
    // ---------------- producer: lane w feeds consumer warp w ----------------
    const int w = lane;
    const int tot = w < NCW ? warp_total(w) : 0;
    const int pw = w < NCW ? ctrl[8 + w] : 0;   // positions issued so far
    const int p0 = changed ? pw : 0;            // position of stage 0
    int iss = changed ? 0 : pw;                 // next stage to issue
    const uint64_t pol = l2_policy_evict_first();
    uint64_t t_idle = globaltimer_ns();
    while (__any_sync(0xffffffffu, iss < tot)) {
      bool progress = false;
      if (iss < tot) {
        const int pos = p0 + iss;
        const int slot = w * depth + pos % depth;
        if (mbar_test(&empty[slot], ((uint32_t)(pos / depth) & 1u) ^ 1u)) {
          const int j = w + iss * NCW;
          const int g = j / cpg;
          const int ch = j - g * cpg;
          const int nr = min(RC, nrows - ch * RC);
          const int e = max(r.sg_exp[g], 0);
          uint8_t* st = ring + (size_t)slot * SB;
          const size_t row0 = (size_t)e * a.H + r0 + ch * RC;
          uint32_t tx = (uint32_t)(nr * row_bytes);
          if constexpr (FMT == W_E4M3) {
            const uintptr_t s0 = (uintptr_t)(a.wscale + row0 * (I / 32));
            const uintptr_t s1 = s0 + (uintptr_t)nr * (I / 32);
            const uint8_t* s_src = (const uint8_t*)(s0 & ~(uintptr_t)15);
            const uint32_t s_len = (uint32_t)(((s1 + 15) & ~(uintptr_t)15) - (uintptr_t)s_src);
            mbar_arrive_expect_tx(&full[slot], tx + s_len);
            bulk_g2s(st + sc_off, s_src, s_len, &full[slot], pol);
          } else {
            mbar_arrive_expect_tx(&full[slot], tx);
          }
          bulk_g2s(st, a.w + row0 * row_bytes, tx, &full[slot], pol);
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
    if (w < NCW) ctrl[8 + w] = p0 + iss;
  } else {
    // ---------------- consumers ----------------
    const int lpr = a.lpr;
    const int rpp = 32 / lpr;  // rows per pass of the warp
    const int prow = lane / lpr;
    const int lj = lane - prow * lpr;
    const int nvec = I / EPV;
    float* my_tile = tiles + (size_t)warp * tile;
    const bool hsm = a.h_smem != 0;
    const __nv_bfloat16* hbase = hsm ? hs : a.h;
    int pos = 0;
    // Stale prefetched stages (routing changed): take them off the ring.
    for (; pos < pos0; ++pos) {
      const int slot = warp * depth + pos % depth;
      if (!mbar_wait(&full[slot], (uint32_t)(pos / depth) & 1u)) {
        ctrl[0] = 1;
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (a.h_smem && !mbar_wait(hbar, 0)) {
      if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
    const int total = warp_total(warp);
    for (int s = 0; s < total; ++s, ++pos) {
      const int j = warp + s * NCW;
      const int g = j / cpg;
      const int ch = j - g * cpg;
      const int lr0 = ch * RC;
      const int nr = min(RC, nrows - lr0);
      const int e = r.sg_exp[g];
      const int cnt = r.sg_cnt[g];
      const int beg = r.sg_beg[g];
      const int slot = warp * depth + pos % depth;
      if (ctrl[0] || !mbar_wait(&full[slot], (uint32_t)(pos / depth) & 1u)) {
        if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
        ctrl[0] = 1;
        break;
      }
      if (e >= 0) {  // a slot with an out-of-range expert id contributes nothing
        const uint8_t* st = ring + (size_t)slot * SB;
        const uint8_t* sbase = nullptr;
        if constexpr (FMT == W_E4M3) {
          const uintptr_t s0 = (uintptr_t)(a.wscale + ((size_t)e * a.H + r0 + lr0) * (I / 32));
          sbase = st + sc_off + (s0 & 15);
        }
        if (cnt == 1)
          dn_item<FMT, 1>(st, sbase, row_bytes, I / 32, nr, nvec, lpr, rpp, prow, lj, r, beg,
                          cnt, hbase, hsm, I, s_scale, my_tile, a.rows_max, lr0);
        else if (cnt == 2)
          dn_item<FMT, 2>(st, sbase, row_bytes, I / 32, nr, nvec, lpr, rpp, prow, lj, r, beg,
                          cnt, hbase, hsm, I, s_scale, my_tile, a.rows_max, lr0);
        else if (cnt <= 4)
          dn_item<FMT, 4>(st, sbase, row_bytes, I / 32, nr, nvec, lpr, rpp, prow, lj, r, beg,
                          cnt, hbase, hsm, I, s_scale, my_tile, a.rows_max, lr0);
        else
          dn_item<FMT, GROUP_MAX>(st, sbase, row_bytes, I / 32, nr, nvec, lpr, rpp, prow, lj, r,
                                  beg, cnt, hbase, hsm, I, s_scale, my_tile, a.rows_max, lr0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // slot back to the producer
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
    const size_t o = (size_t)b * a.H + r0 + lr;
    if (a.out_fp32)
      reinterpret_cast<float*>(a.out)[o] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(v);
  }
}

}  // namespace wdb
