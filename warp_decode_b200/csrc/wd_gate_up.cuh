// gate_up + silu_and_mul for MoE decode, sm_100a.
//
// Computes, for every slot i = b*topk + s with expert e = topk_ids[b, s]:
//   h[i, n] = silu(x[b] . W[e, n, :]) * (x[b] . W[e, inter + n, :])
// (the operation of moe_gate_up_3d_batched_kernel,
//  csrc/moe_gate_up_3d_batched.cu:49-115 of the reference).
//
// Design (B200):
//  * Persistent grid, one CTA per SM: 8 consumer warps + 1 producer warp.
//    The work list is (group, neuron) items, a group being up to GROUP_MAX
//    slots that share an expert: a weight row is streamed from HBM once per
//    call however many tokens of the batch picked that expert (the reference
//    re-reads it per slot).  Items go to consumer warps round-robin.
//  * Every consumer warp owns `depth` ring slots.  Lane w of the producer warp
//    feeds consumer warp w: it polls that warp's "empty" mbarriers without
//    blocking and issues cp.async.bulk copies of the gate and up row chunks
//    (up to 4 KB each) into the freed slot, completing the slot's "full" mbarrier
//    by byte count.  The 8 lanes issue in parallel, so copy issue never sits
//    on a consumer's critical path, and a slot is only ever consumed, in
//    order, by one warp.
//  * x of the whole batch is bulk-copied into shared memory once per CTA.
//    Consumers read 16-byte weight and activation vectors from shared memory
//    and accumulate with bf16-input / FP32-accumulate FMAs; a butterfly
//    reduction and the fused silu(g)*u epilogue finish the item.
//  * The grid signals programmatic launch completion at entry, so a directly
//    following down kernel can become resident and prefetch its weights while
//    this one still streams.
#pragma once

#include <cuda_fp8.h>

#include "wd_common.cuh"

namespace wdb {

enum WFmt : int { W_BF16 = 0, W_E4M3 = 1 };

struct GateUpArgs {
  const __nv_bfloat16* x;   // [B, H]
  const uint8_t* w;         // [E, 2I, H] bf16 or e4m3
  const uint8_t* wscale;    // [E, 2I, H/32] ue8m0 (e4m3 only)
  const int32_t* ids;       // [B, K]
  __nv_bfloat16* out;       // [B*K, I]
  uint32_t* status;
  int B, E, K, H, I;
  int dedup;
  int kc;           // weight elements per row chunk (multiple of 512)
  int depth;        // ring slots per consumer warp
  int stage_bytes;  // bytes per ring slot (multiple of 128)
  int x_smem;       // 1: x staged in shared memory
};

constexpr int GU_THREADS = (NWARPS + 1) * 32;
// Control words after the barriers: [0] abort flag, [8+w] stages issued for
// consumer warp w, [16+w] stages consumed by it.
constexpr int CTRL_INTS = 32;

template <int FMT>
struct GuFmt {
  static constexpr int WB = FMT == W_BF16 ? 2 : 1;   // bytes per weight
};

// Scale bytes of one row chunk, copied from a 16-byte aligned start (so up to
// 30 bytes of slack), rounded to 16.
__host__ __device__ inline int gate_up_scale_slot(int kc) { return ((kc / 32 + 32 + 15) / 16) * 16; }

// Bytes of one ring slot: gate chunk, up chunk (+ their scale bytes).
__host__ __device__ inline int gate_up_stage_bytes(int fmt, int kc) {
  const int wb = fmt == W_BF16 ? 2 : 1;
  const int sc = fmt == W_E4M3 ? gate_up_scale_slot(kc) : 0;
  return ((2 * kc * wb + 2 * sc + 127) / 128) * 128;
}

__host__ inline int gate_up_smem_bytes(int depth, int stage_bytes, int x_bytes, int n, int E,
                                       bool dedup) {
  return NWARPS * depth * stage_bytes + ((x_bytes + 127) / 128) * 128 +
         (2 * NWARPS * depth + 1) * 8 + CTRL_INTS * 4 + route_smem_bytes(n, E, dedup);
}

__device__ __forceinline__ float silu_f32(float v) { return v / (1.0f + __expf(-v)); }

// 16-byte activation vector: shared-memory tile or global memory.
__device__ __forceinline__ uint4 act16(const __nv_bfloat16* p, bool smem) {
  return smem ? lds16(p) : ldg16(p);
}

// One chunk of one item: accumulate x[tok[m]] . gate / up over this chunk
// into two partial sums each (ag/ag2, au/au2: shorter dependency chains).
// MAXM bounds the member count at compile time (registers stay static).
template <int FMT, int MAXM>
__device__ __forceinline__ void gu_chunk(const uint8_t* __restrict__ gs,
                                         const uint8_t* __restrict__ us, const uint8_t* gsc,
                                         const uint8_t* usc, int klen,
                                         const __nv_bfloat16* const (&xr)[GROUP_MAX], bool xsm,
                                         int cnt, int lane, float (&ag)[GROUP_MAX],
                                         float (&ag2)[GROUP_MAX], float (&au)[GROUP_MAX],
                                         float (&au2)[GROUP_MAX]) {
  if constexpr (FMT == W_BF16) {
#pragma unroll 2
    for (int k = lane * 8; k < klen; k += 256) {
      const uint4 gv = lds16(gs + k * 2);
      const uint4 uv = lds16(us + k * 2);
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < cnt) {
          const uint4 xv = act16(xr[m] + k, xsm);
          dot8_bf16(ag[m], ag2[m], xv, gv);
          dot8_bf16(au[m], au2[m], xv, uv);
        }
      }
    }
  } else {
    // E4M3: decoded to exact bf16 patterns (scaled by 2^-120), the bf16 FMA,
    // then 2^120 x the block scale once per lane and block.  Not unrolled:
    // registers stay within the two-CTAs-per-SM budget.
#pragma unroll 1
    for (int k = lane * 16; k < klen; k += 512) {
      uint32_t gw[8], uw[8];
      const bool gnan = e4m3x16_to_bf16(lds16(gs + k), gw);
      const bool unan = e4m3x16_to_bf16(lds16(us + k), uw);
      const uint32_t sg = gsc[k >> 5];
      const uint32_t su = usc[k >> 5];
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < cnt) {
          const uint4 xa = act16(xr[m] + k, xsm);
          const uint4 xb = act16(xr[m] + k + 8, xsm);
          float g = 0.f, g2 = 0.f, u = 0.f, u2 = 0.f;
          dot16_e4m3(g, g2, xa, xb, gw);
          dot16_e4m3(u, u2, xa, xb, uw);
          ag[m] = mx_block_fma(g, sg, gnan, ag[m]);
          ag2[m] = mx_block_fma(g2, sg, gnan, ag2[m]);
          au[m] = mx_block_fma(u, su, unan, au[m]);
          au2[m] = mx_block_fma(u2, su, unan, au2[m]);
        }
      }
    }
  }
}

template <int FMT, int kRoute>
__global__ void __maxnreg__(FMT == W_E4M3 ? 96 : 112) moe_gate_up_kernel(const GateUpArgs a) {
  using F = GuFmt<FMT>;
  constexpr int NCW = NWARPS;


  extern __shared__ __align__(128) uint8_t smem[];
  const int depth = a.depth;
  const int SB = a.stage_bytes;
  const int nslots = NCW * depth;
  const size_t H = (size_t)a.H;
  const uint32_t x_bytes = (uint32_t)((size_t)a.B * H * 2);
  uint8_t* ring = smem;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ring + (size_t)nslots * SB);
  uint8_t* after_x =
      reinterpret_cast<uint8_t*>(xs) + (a.x_smem ? ((x_bytes + 127) / 128) * 128 : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(after_x);
  uint64_t* empty = full + nslots;
  uint64_t* xbar = empty + nslots;
  volatile int* ctrl = reinterpret_cast<int*>(xbar + 1);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;

  const int n = a.B * a.K;
  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Barriers initialised in parallel; the x tile copy starts at once.
  if (threadIdx.x < nslots) {
    mbar_init(&full[threadIdx.x], 1);
    mbar_init(&empty[threadIdx.x], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 32 * NCW) {
    mbar_init(xbar, 1);
    ctrl[0] = 0;
    fence_mbar_init();
    if (a.x_smem) {
      mbar_arrive_expect_tx(xbar, x_bytes);
      bulk_g2s_big(xs, a.x, x_bytes, xbar, l2_policy_evict_last());
    }
  }
  route_build<false, NoInit, kRoute>(r, a.ids, n, a.E, a.K, dedup, GROUP_MAX,
                                     a.status);  // ends with __syncthreads

  const int nsg = *r.nsg;
  const int items = nsg * a.I;  // host guarantees n * I < 2^31
  const int KC = a.kc;
  const int nchunks = (a.H + KC - 1) / KC;
  const int G = (int)gridDim.x;
  const int cta_items = items > (int)blockIdx.x ? (items - (int)blockIdx.x + G - 1) / G : 0;
  const int sc_slot = FMT == W_E4M3 ? gate_up_scale_slot(KC) : 0;
  auto warp_total = [&](int w) {
    const int wi = cta_items > w ? (cta_items - w + NCW - 1) / NCW : 0;
    return wi * nchunks;
  };
  // Stage s of consumer warp w: its il-th item (il = s / nchunks), chunk c.
  auto stage_item = [&](int w, int s, int& c, int& sg, int& nn) {
    const int il = s / nchunks;
    c = s - il * nchunks;
    const int t = (int)blockIdx.x + (w + il * NCW) * G;
    sg = t / a.I;
    nn = t - sg * a.I;
  };

  if (warp == NCW) {
    // ---------------- producer: lane w feeds consumer warp w ----------------
    const int w = lane;
    const int tot = w < NCW ? warp_total(w) : 0;
    const uint64_t pol = l2_policy_evict_first();
    int iss = 0;
    uint64_t t_idle = globaltimer_ns();
    while (__any_sync(0xffffffffu, iss < tot)) {
      bool progress = false;
      if (iss < tot) {
        const int slot = w * depth + iss % depth;
        if (mbar_test(&empty[slot], ((uint32_t)(iss / depth) & 1u) ^ 1u)) {
          int c, sg, nn;
          stage_item(w, iss, c, sg, nn);
          const int e = max(r.sg_exp[sg], 0);  // invalid-id group: any valid rows
          uint8_t* st = ring + (size_t)slot * SB;
          const int kc = c * KC;
          const int klen = min(KC, a.H - kc);
          const size_t row_g = (size_t)e * 2 * a.I + nn;
          const size_t row_u = row_g + a.I;
          const uint32_t wbytes = (uint32_t)klen * F::WB;
          uint32_t tx = 2 * wbytes;
          const uint8_t* sg_src = nullptr;
          const uint8_t* su_src = nullptr;
          uint32_t sg_len = 0, su_len = 0;
          if constexpr (FMT == W_E4M3) {
            // Scale bytes of this chunk, copied from a 16-byte aligned start.
            const uintptr_t g0 = (uintptr_t)(a.wscale + (row_g * H + kc) / 32);
            const uintptr_t u0 = (uintptr_t)(a.wscale + (row_u * H + kc) / 32);
            const uintptr_t len = (uintptr_t)klen / 32;
            sg_src = (const uint8_t*)(g0 & ~(uintptr_t)15);
            su_src = (const uint8_t*)(u0 & ~(uintptr_t)15);
            sg_len = (uint32_t)(((g0 + len + 15) & ~(uintptr_t)15) - (uintptr_t)sg_src);
            su_len = (uint32_t)(((u0 + len + 15) & ~(uintptr_t)15) - (uintptr_t)su_src);
            tx += sg_len + su_len;
          }
          mbar_arrive_expect_tx(&full[slot], tx);
          bulk_g2s(st, a.w + (row_g * H + kc) * F::WB, wbytes, &full[slot], pol);
          bulk_g2s(st + (size_t)KC * F::WB, a.w + (row_u * H + kc) * F::WB, wbytes, &full[slot],
                   pol);
          if constexpr (FMT == W_E4M3) {
            bulk_g2s(st + 2 * (size_t)KC, sg_src, sg_len, &full[slot], pol);
            bulk_g2s(st + 2 * (size_t)KC + sc_slot, su_src, su_len, &full[slot], pol);
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
    // ---------------- consumers ----------------
    const int total = warp_total(warp);
    if (a.x_smem && !mbar_wait(xbar, 0)) {
      if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      ctrl[0] = 1;
    }
    float ag[GROUP_MAX], ag2[GROUP_MAX], au[GROUP_MAX], au2[GROUP_MAX];
    const __nv_bfloat16* xrow[GROUP_MAX];
    int cnt = 0, beg = 0, e = 0;
    int s = 0;
    for (; s < total; ++s) {
      int c, sg, nn;
      stage_item(warp, s, c, sg, nn);
      if (c == 0) {
        e = r.sg_exp[sg];
        cnt = r.sg_cnt[sg];
        beg = r.sg_beg[sg];
#pragma unroll
        for (int m = 0; m < GROUP_MAX; ++m) {
          const int tok = r.mtok[beg + (m < cnt ? m : 0)];
          xrow[m] = (a.x_smem ? xs : a.x) + (size_t)tok * H;
          ag[m] = 0.f;
          ag2[m] = 0.f;
          au[m] = 0.f;
          au2[m] = 0.f;
        }
      }
      const int slot = warp * depth + s % depth;
      if (ctrl[0] || !mbar_wait(&full[slot], (uint32_t)(s / depth) & 1u)) {
        if (lane == 0) raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
        ctrl[0] = 1;
        break;
      }
      if (e >= 0) {
        const uint8_t* st = ring + (size_t)slot * SB;
        const int kc = c * KC;
        const int klen = min(KC, a.H - kc);
        const uint8_t* gsc = nullptr;
        const uint8_t* usc = nullptr;
        if constexpr (FMT == W_E4M3) {
          const size_t row_g = (size_t)e * 2 * a.I + nn;
          const uintptr_t g0 = (uintptr_t)(a.wscale + (row_g * H + kc) / 32);
          const uintptr_t u0 = (uintptr_t)(a.wscale + ((row_g + a.I) * H + kc) / 32);
          gsc = st + 2 * (size_t)KC + (g0 & 15);
          usc = st + 2 * (size_t)KC + sc_slot + (u0 & 15);
        }
        const __nv_bfloat16* xr[GROUP_MAX];
#pragma unroll
        for (int m = 0; m < GROUP_MAX; ++m) xr[m] = xrow[m] + kc;
        const uint8_t* gs = st;
        const uint8_t* us = st + (size_t)KC * F::WB;
        const bool xsm = a.x_smem != 0;
        if (cnt == 1)
          gu_chunk<FMT, 1>(gs, us, gsc, usc, klen, xr, xsm, cnt, lane, ag, ag2, au, au2);
        else if (cnt == 2)
          gu_chunk<FMT, 2>(gs, us, gsc, usc, klen, xr, xsm, cnt, lane, ag, ag2, au, au2);
        else if (cnt <= 4)
          gu_chunk<FMT, 4>(gs, us, gsc, usc, klen, xr, xsm, cnt, lane, ag, ag2, au, au2);
        else
          gu_chunk<FMT, GROUP_MAX>(gs, us, gsc, usc, klen, xr, xsm, cnt, lane, ag, ag2, au, au2);
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
              const int slot_i = r.members[beg + m];
              // A slot with an out-of-range expert id yields zeros.
              a.out[(size_t)slot_i * a.I + nn] =
                  __float2bfloat16_rn(e >= 0 ? silu_f32(g) * u : 0.f);
            }
          }
        }
      }
    }
    if (lane == 0) ctrl[16 + warp] = s;
  }
  __syncthreads();
  // This CTA's h rows are written: a directly following down kernel launched
  // with programmatic dependence may start once every CTA got here (it waits
  // for this grid to finish before reading h).  Triggered at entry instead,
  // the down grid launched early, could not take an SM until gate_up CTAs
  // left (shared memory) and started later, not sooner.
  if (threadIdx.x == 0) pdl_launch_dependents();
  // After an abort, let every issued but unconsumed copy land before exit.
  if (ctrl[0] && warp < NCW && lane == 0) {
    for (int q = ctrl[16 + warp]; q < ctrl[8 + warp]; ++q)
      if (!mbar_wait(&full[warp * depth + q % depth], (uint32_t)(q / depth) & 1u)) break;
  }
}

}  // namespace wdb
