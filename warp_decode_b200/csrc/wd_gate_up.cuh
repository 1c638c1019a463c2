// gate_up + silu_and_mul for MoE decode, sm_100a.
//
// Computes, for every slot i = b*topk + s with expert e = topk_ids[b, s]:
//   h[i, n] = silu(x[b] . W[e, n, :]) * (x[b] . W[e, inter + n, :])
// (the operation of moe_gate_up_3d_batched_kernel,
//  csrc/moe_gate_up_3d_batched.cu:49-115 of the reference).
//
// Design (B200):
//  * Persistent grid, one CTA per SM.  The work list is (group, neuron)
//    items where a group is up to GROUP_MAX slots sharing an expert, so a
//    weight row is streamed from HBM once per call however many tokens of the
//    batch picked that expert (the reference re-reads it per slot).
//  * One producer thread streams the gate row and the up row of each item
//    (chunks of up to 4 KB each, one 8 KB stage per chunk pair) with
//    cp.async.bulk into shared memory.  Items go to the eight consumer warps
//    round-robin and every warp owns a private 2-slot ring (16 slots in all,
//    mbarriers full: bytes landed / empty: consumer done), which it alone
//    consumes in order.
//  * Each consumer warp computes its items whole: each lane reads
//    16-byte weight vectors from shared memory, the matching activation
//    vectors of every group member from global memory (L1-resident), and
//    accumulates FP32 dot products; a butterfly reduction and the fused
//    silu(g)*u epilogue finish the item.
//  * The grid signals programmatic launch completion at entry, so a directly
//    following down kernel can become resident and prefetch its weights
//    while this one still streams.
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
};

constexpr int GU_CONSUMER_WARPS = 8;
constexpr int GU_DEPTH = 2;  // ring slots per consumer warp
constexpr int GU_STAGES = GU_CONSUMER_WARPS * GU_DEPTH;
constexpr int GU_THREADS = (GU_CONSUMER_WARPS + 1) * 32;

template <int FMT>
struct GateUpCfg {
  static constexpr int WB = (FMT == W_BF16) ? 2 : 1;        // bytes per weight
  static constexpr int KC = 4096 / WB;                      // elements per chunk
  static constexpr int ROW_BYTES = KC * WB;                 // 4 KB
  static constexpr int SC_BYTES = (FMT == W_E4M3) ? (KC / 32 + 32) : 0;
  static constexpr int STAGE_BYTES = ((2 * ROW_BYTES + 2 * SC_BYTES + 127) / 128) * 128;
};

__host__ inline int gate_up_smem_bytes(int fmt, int n, int E, bool dedup) {
  const int stage = fmt == W_BF16 ? GateUpCfg<W_BF16>::STAGE_BYTES : GateUpCfg<W_E4M3>::STAGE_BYTES;
  return GU_STAGES * stage + 2 * GU_STAGES * 8 + 16 + route_smem_bytes(n, E, dedup);
}

__device__ __forceinline__ float silu_f32(float v) { return v / (1.0f + __expf(-v)); }

// Dot products of one 16-byte weight vector pair against member activations.
template <int FMT>
struct GateUpMath;

template <>
struct GateUpMath<W_BF16> {
  static constexpr int EPV = 8;  // elements per 16-byte vector
  // gs/us: stage pointers of this chunk; k: element offset in chunk.
  __device__ __forceinline__ static void step(const uint8_t* gs, const uint8_t* us,
                                              const uint8_t* /*gsc*/, const uint8_t* /*usc*/,
                                              int k, const __nv_bfloat16* const (&xrow)[GROUP_MAX],
                                              int kglob, int cnt, float (&ag)[GROUP_MAX],
                                              float (&au)[GROUP_MAX]) {
    float gf[8], uf[8];
    unpack_bf16x8(lds16(gs + k * 2), gf);
    unpack_bf16x8(lds16(us + k * 2), uf);
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt) {
        float xf[8];
        unpack_bf16x8(ldg16(xrow[m] + kglob), xf);
        float g = ag[m], u = au[m];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          g = fmaf(xf[t], gf[t], g);
          u = fmaf(xf[t], uf[t], u);
        }
        ag[m] = g;
        au[m] = u;
      }
    }
  }
};

__device__ __forceinline__ void unpack_e4m3x16(const uint4& v, float (&f)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[q] & 0xffffu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[q] >> 16), __NV_E4M3);
    const float2 a = __half22float2(__half2(lo));
    const float2 b = __half22float2(__half2(hi));
    f[4 * q + 0] = a.x; f[4 * q + 1] = a.y;
    f[4 * q + 2] = b.x; f[4 * q + 3] = b.y;
  }
}

template <>
struct GateUpMath<W_E4M3> {
  static constexpr int EPV = 16;
  __device__ __forceinline__ static void step(const uint8_t* gs, const uint8_t* us,
                                              const uint8_t* gsc, const uint8_t* usc, int k,
                                              const __nv_bfloat16* const (&xrow)[GROUP_MAX],
                                              int kglob, int cnt, float (&ag)[GROUP_MAX],
                                              float (&au)[GROUP_MAX]) {
    float gf[16], uf[16];
    unpack_e4m3x16(lds16(gs + k), gf);
    unpack_e4m3x16(lds16(us + k), uf);
    const float sg = ue8m0_to_f32(gsc[k >> 5]);
    const float su = ue8m0_to_f32(usc[k >> 5]);
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt) {
        float xf[16];
        float xa[8], xb[8];
        unpack_bf16x8(ldg16(xrow[m] + kglob), xa);
        unpack_bf16x8(ldg16(xrow[m] + kglob + 8), xb);
#pragma unroll
        for (int t = 0; t < 8; ++t) { xf[t] = xa[t]; xf[8 + t] = xb[t]; }
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          g = fmaf(xf[t], gf[t], g);
          u = fmaf(xf[t], uf[t], u);
        }
        ag[m] = fmaf(g, sg, ag[m]);
        au[m] = fmaf(u, su, au[m]);
      }
    }
  }
};

template <int FMT>
__global__ void __launch_bounds__(GU_THREADS, 2) moe_gate_up_kernel(const GateUpArgs a) {
  using Cfg = GateUpCfg<FMT>;
  using Math = GateUpMath<FMT>;
  constexpr int KC = Cfg::KC;
  constexpr int NCW = GU_CONSUMER_WARPS;
  constexpr int D = GU_DEPTH;

  // Let a directly following down kernel start its prologue now.
  pdl_launch_dependents();

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GU_STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + GU_STAGES;
  int* abort_flag = reinterpret_cast<int*>(empty + GU_STAGES);
  int* route_base = abort_flag + 4;

  const int n = a.B * a.K;
  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GU_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  build_groups(r, a.ids, n, a.E, dedup, a.status);  // ends with __syncthreads

  const int nsg = *r.nsg;
  const long long items = (long long)nsg * a.I;
  const int nchunks = (a.H + KC - 1) / KC;
  const size_t H = (size_t)a.H;

  // Item j of this CTA belongs to consumer warp j % NCW.  Every consumer warp
  // owns D ring slots (slots w*D .. w*D+D-1) that only it consumes, in
  // order, so a parity wait never runs more than one phase ahead.
  if (warp == NCW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int tw[NCW];
#pragma unroll
      for (int w = 0; w < NCW; ++w) tw[w] = 0;
      bool ok = true;
      int j = 0;
      for (long long t = blockIdx.x; t < items && ok; t += gridDim.x, ++j) {
        const int sg = (int)(t / a.I);
        const int nn = (int)(t - (long long)sg * a.I);
        const int e = r.sg_exp[sg];
        if (e < 0) continue;
        const int w = j % NCW;
        const size_t row_g = (size_t)e * 2 * a.I + nn;
        const size_t row_u = row_g + a.I;
        for (int c = 0; c < nchunks; ++c) {
          const int kc = c * KC;
          const int klen = min(KC, a.H - kc);
          const int tt = tw[w]++;
          const int slot = w * D + tt % D;
          const uint32_t ph = (uint32_t)(tt / D) & 1u;
          if (!mbar_wait(&empty[slot], ph ^ 1u) || *(volatile int*)abort_flag) {
            *(volatile int*)abort_flag = 1;
            raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
            tw[w]--;  // this stage was never issued
            ok = false;
            break;
          }
          uint8_t* st = stages + slot * Cfg::STAGE_BYTES;
          const uint32_t wbytes = (uint32_t)klen * Cfg::WB;
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
            sg_len = (uint32_t)((((g0 + len) + 15) & ~(uintptr_t)15) - (uintptr_t)sg_src);
            su_len = (uint32_t)((((u0 + len) + 15) & ~(uintptr_t)15) - (uintptr_t)su_src);
            tx += sg_len + su_len;
          }
          mbar_arrive_expect_tx(&full[slot], tx);
          bulk_g2s(st, a.w + (row_g * H + kc) * Cfg::WB, wbytes, &full[slot], pol);
          bulk_g2s(st + Cfg::ROW_BYTES, a.w + (row_u * H + kc) * Cfg::WB, wbytes, &full[slot], pol);
          if constexpr (FMT == W_E4M3) {
            bulk_g2s(st + 2 * Cfg::ROW_BYTES, sg_src, sg_len, &full[slot], pol);
            bulk_g2s(st + 2 * Cfg::ROW_BYTES + Cfg::SC_BYTES, su_src, su_len, &full[slot], pol);
          }
        }
      }
      // Drain: no copy may still be landing in shared memory when we exit.
      for (int w = 0; w < NCW && ok; ++w) {
        for (int tt = max(0, tw[w] - D); tt < tw[w]; ++tt) {
          if (!mbar_wait(&full[w * D + tt % D], (uint32_t)(tt / D) & 1u)) {
            raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  int tt = 0;  // this warp's stage counter
  int j = 0;
  for (long long t = blockIdx.x; t < items; t += gridDim.x, ++j) {
    if ((j % NCW) != warp) continue;
    const int sg = (int)(t / a.I);
    const int nn = (int)(t - (long long)sg * a.I);
    const int e = r.sg_exp[sg];
    const int cnt = r.sg_cnt[sg];
    const int beg = r.sg_beg[sg];
    if (e < 0) {
      // Slots with an invalid expert id produce zeros.
      if (lane < cnt) {
        const int slot_i = r.members[beg + lane];
        a.out[(size_t)slot_i * a.I + nn] = __float2bfloat16_rn(0.f);
      }
      continue;
    }
    if (*(volatile int*)abort_flag) break;

    const __nv_bfloat16* xrow[GROUP_MAX];
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      const int slot_i = m < cnt ? r.members[beg + m] : r.members[beg];
      xrow[m] = a.x + (size_t)(slot_i / a.K) * H;
    }
    float ag[GROUP_MAX], au[GROUP_MAX];
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) { ag[m] = 0.f; au[m] = 0.f; }

    bool ok = true;
    for (int c = 0; c < nchunks; ++c, ++tt) {
      const int kc = c * KC;
      const int klen = min(KC, a.H - kc);
      const int slot = warp * D + tt % D;
      if (!mbar_wait(&full[slot], (uint32_t)(tt / D) & 1u)) {
        ok = false;
        break;
      }
      const uint8_t* st = stages + slot * Cfg::STAGE_BYTES;
      const uint8_t* gs = st;
      const uint8_t* us = st + Cfg::ROW_BYTES;
      const uint8_t* gsc = nullptr;
      const uint8_t* usc = nullptr;
      if constexpr (FMT == W_E4M3) {
        // Offsets of this chunk's scales inside the aligned copies.
        const size_t row_g = (size_t)e * 2 * a.I + nn;
        const size_t row_u = row_g + a.I;
        const uintptr_t g0 = (uintptr_t)(a.wscale + (row_g * H + kc) / 32);
        const uintptr_t u0 = (uintptr_t)(a.wscale + (row_u * H + kc) / 32);
        gsc = st + 2 * Cfg::ROW_BYTES + (g0 & 15);
        usc = st + 2 * Cfg::ROW_BYTES + Cfg::SC_BYTES + (u0 & 15);
      }
#pragma unroll 2
      for (int k = lane * Math::EPV; k < klen; k += 32 * Math::EPV) {
        Math::step(gs, us, gsc, usc, k, xrow, kc + k, cnt, ag, au);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (!ok) {
      if (lane == 0) {
        *(volatile int*)abort_flag = 1;
        raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      }
      break;
    }
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt) {
        ag[m] = warp_sum(ag[m]);
        au[m] = warp_sum(au[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt && lane == m) {
        const int slot_i = r.members[beg + m];
        a.out[(size_t)slot_i * a.I + nn] = __float2bfloat16_rn(silu_f32(ag[m]) * au[m]);
      }
    }
  }
}

}  // namespace wdb
