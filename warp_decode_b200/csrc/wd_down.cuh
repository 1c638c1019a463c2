// down projection + top-k weighted sum for MoE decode, sm_100a.
//
// Computes y[b, j] = sum_s topk_scale[b,s] * (h[b*topk+s, :] . Wd[e_s, j, :])
// (the operation of moe_down_3d_batched_kernel,
//  csrc/moe_down_3d_batched.cu:45-122 of the reference), with FP32 products
// and FP32 accumulation (the reference rounds each product to bf16 first).
//
// Design (B200):
//  * Persistent grid, one CTA per SM.  CTA c owns output rows
//    [c*H/G, (c+1)*H/G) for every token, so the top-k reduction never leaves
//    the CTA: no atomics, no second pass, no scratch memory.
//  * For each routing group (up to GROUP_MAX slots sharing an expert) the
//    CTA's rows of that expert form one contiguous block of Wd; the producer
//    thread streams it in stages of up to ~12 KB with cp.async.bulk into an
//    NS-deep ring.  Each expert's rows are read from HBM once per call.
//  * Consumer warps own fixed quads of rows (8 lanes per row, 16-byte
//    vectors); per stage they dot every member's activation row (L1-resident)
//    against the staged weight rows and add scale * dot into a per-CTA FP32
//    accumulator tile [B][rows] in shared memory, written only by the owner.
//  * Programmatic dependent launch: routing and the first NS weight stages
//    are issued before griddepcontrol.wait, i.e. while a preceding gate_up
//    grid still runs.  h and topk_scale are read only after the wait.  A
//    verifier warp re-reads topk_ids after the wait; if they differ from
//    what the prologue saw, the whole pass is redone with the new routing.
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
  int nstages;
  int stage_rows;           // rows per stage (multiple of 4 unless rows/CTA < 4)
  int rows_max;             // max rows per CTA (ceil(H / gridDim.x))
  int stage_bytes;          // bytes per ring slot (weights + scales), multiple of 128
};

constexpr int DN_CONSUMER_WARPS = 8;
constexpr int DN_THREADS = (DN_CONSUMER_WARPS + 2) * 32;  // + producer + verifier
constexpr int DN_STAGE_TARGET = 12 * 1024;

template <int FMT>
__host__ __device__ inline int down_scale_area(int stage_rows, int I) {
  return FMT == W_E4M3 ? ((stage_rows * (I / 32) + 32 + 15) / 16) * 16 : 0;
}

__host__ inline int down_smem_bytes(int nstages, int stage_bytes, int B, int rows_max, int n, int E,
                                    bool dedup) {
  return nstages * stage_bytes + 2 * nstages * 8 + 16 + B * rows_max * 4 +
         route_smem_bytes(n, E, dedup);
}

template <int FMT>
struct DownMath;

template <>
struct DownMath<W_BF16> {
  static constexpr int EPV = 8;
  // One 16-byte weight vector against every member's matching activations.
  __device__ __forceinline__ static void step(const uint8_t* wrow, const uint8_t* /*srow*/, int v,
                                              const __nv_bfloat16* const (&hrow)[GROUP_MAX],
                                              int cnt, float (&acc)[GROUP_MAX]) {
    float wf[8];
    unpack_bf16x8(lds16(wrow + v * 16), wf);
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt) {
        float hf[8];
        unpack_bf16x8(ldg16(hrow[m] + v * 8), hf);
        float s = acc[m];
#pragma unroll
        for (int t = 0; t < 8; ++t) s = fmaf(hf[t], wf[t], s);
        acc[m] = s;
      }
    }
  }
};

template <>
struct DownMath<W_E4M3> {
  static constexpr int EPV = 16;
  __device__ __forceinline__ static void step(const uint8_t* wrow, const uint8_t* srow, int v,
                                              const __nv_bfloat16* const (&hrow)[GROUP_MAX],
                                              int cnt, float (&acc)[GROUP_MAX]) {
    float wf[16];
    unpack_e4m3x16(lds16(wrow + v * 16), wf);
    const float sc = ue8m0_to_f32(srow[v >> 1]);
#pragma unroll
    for (int m = 0; m < GROUP_MAX; ++m) {
      if (m < cnt) {
        float ha[8], hb[8];
        unpack_bf16x8(ldg16(hrow[m] + v * 16), ha);
        unpack_bf16x8(ldg16(hrow[m] + v * 16 + 8), hb);
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < 8; ++t) s = fmaf(ha[t], wf[t], s);
#pragma unroll
        for (int t = 0; t < 8; ++t) s = fmaf(hb[t], wf[8 + t], s);
        acc[m] = fmaf(s, sc, acc[m]);
      }
    }
  }
};

template <int FMT>
__global__ void __launch_bounds__(DN_THREADS, 2) moe_down_kernel(const DownArgs a) {
  using Math = DownMath<FMT>;
  constexpr int WB = (FMT == W_BF16) ? 2 : 1;

  extern __shared__ __align__(128) uint8_t smem[];
  const int NS = a.nstages;
  const int SB = a.stage_bytes;
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  int* flags = reinterpret_cast<int*>(empty + NS);  // [0] abort, [1] routing changed
  float* acc_tile = reinterpret_cast<float*>(flags + 4);
  int* route_base = reinterpret_cast<int*>(acc_tile + a.B * a.rows_max);

  const int n = a.B * a.K;
  const bool dedup = a.dedup != 0;
  const RouteSmem r = route_carve(route_base, n, a.E, dedup);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = (int)((long long)blockIdx.x * a.H / gridDim.x);
  const int r1 = (int)((long long)(blockIdx.x + 1) * a.H / gridDim.x);
  const int nrows = r1 - r0;
  const int RS = a.stage_rows;
  const int I = a.I;
  const size_t row_bytes = (size_t)I * WB;
  const int nvec = I / Math::EPV;  // 16-byte vectors per weight row
  const int sc_area_off = RS * (int)row_bytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], DN_CONSUMER_WARPS);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < a.B * a.rows_max; i += blockDim.x) acc_tile[i] = 0.f;

  int q = 0;  // ring position, identical in the producer and every consumer
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      // The routing read before the dependency wait was stale: redo.
      if (flags[1] == 0) break;
      pdl_wait_primary();
      for (int i = threadIdx.x; i < a.B * a.rows_max; i += blockDim.x) acc_tile[i] = 0.f;
      if (threadIdx.x == 0) raise_status(a.status, WD_STATUS_ROUTING_CHANGED);
    }
    build_groups(r, a.ids, n, a.E, dedup, a.status);  // ends with __syncthreads
    const int nsg = *r.nsg;

    if (warp == DN_CONSUMER_WARPS) {
      // ---------------- producer ----------------
      if (lane == 0) {
        const uint64_t pol = l2_policy_evict_first();
        bool ok = true;
        const int q0 = q;
        for (int sg = 0; sg < nsg && ok; ++sg) {
          const int e = r.sg_exp[sg];
          if (e < 0) continue;
          for (int rb = r0; rb < r1; rb += RS, ++q) {
            const int nr = min(RS, r1 - rb);
            const int slot = q % NS;
            const uint32_t ph = (uint32_t)(q / NS) & 1u;
            if (!mbar_wait(&empty[slot], ph ^ 1u) || *(volatile int*)&flags[0]) {
              *(volatile int*)&flags[0] = 1;
              raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
              ok = false;
              break;
            }
            uint8_t* st = stages + slot * SB;
            const size_t row0 = (size_t)e * a.H + rb;
            const uint32_t wbytes = (uint32_t)(nr * row_bytes);
            uint32_t tx = wbytes;
            const uint8_t* s_src = nullptr;
            uint32_t s_len = 0;
            if constexpr (FMT == W_E4M3) {
              const uintptr_t s0 = (uintptr_t)(a.wscale + row0 * (I / 32));
              const uintptr_t s1 = s0 + (uintptr_t)nr * (I / 32);
              s_src = (const uint8_t*)(s0 & ~(uintptr_t)15);
              s_len = (uint32_t)(((s1 + 15) & ~(uintptr_t)15) - (uintptr_t)s_src);
              tx += s_len;
            }
            mbar_arrive_expect_tx(&full[slot], tx);
            bulk_g2s(st, a.w + row0 * row_bytes, wbytes, &full[slot], pol);
            if constexpr (FMT == W_E4M3) bulk_g2s(st + sc_area_off, s_src, s_len, &full[slot], pol);
          }
        }
        for (int s = max(q0, q - NS); s < q; ++s) {
          if (!mbar_wait(&full[s % NS], (uint32_t)(s / NS) & 1u)) {
            raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
            break;
          }
        }
      }
      q = __shfl_sync(0xffffffffu, q, 0);
    } else if (warp == DN_CONSUMER_WARPS + 1) {
      // ---------------- verifier ----------------
      if (pass == 0) {
        pdl_wait_primary();
        bool diff = false;
        for (int i = lane; i < n; i += 32) {
          int e = __ldg(a.ids + i);
          if (e < 0 || e >= a.E) e = -1;
          diff |= (e != r.ids[i]);
        }
        if (__any_sync(0xffffffffu, diff) && lane == 0) flags[1] = 1;
      }
    } else {
      // ---------------- consumers ----------------
      pdl_wait_primary();  // h and topk_scale come from the preceding grid
      const int sub = lane >> 3;  // row inside the quad
      const int j8 = lane & 7;    // lane inside the row
      bool ok = true;
      for (int sg = 0; sg < nsg && ok; ++sg) {
        const int e = r.sg_exp[sg];
        if (e < 0) continue;
        const int cnt = r.sg_cnt[sg];
        const int beg = r.sg_beg[sg];
        const __nv_bfloat16* hrow[GROUP_MAX];
        float sc[GROUP_MAX];
        int tok[GROUP_MAX];
#pragma unroll
        for (int m = 0; m < GROUP_MAX; ++m) {
          const int slot_i = m < cnt ? r.members[beg + m] : r.members[beg];
          hrow[m] = a.h + (size_t)slot_i * I;
          sc[m] = __ldg(a.scale + slot_i);
          tok[m] = slot_i / a.K;
        }
        for (int rb = r0; rb < r1; rb += RS, ++q) {
          const int nr = min(RS, r1 - rb);
          const int slot = q % NS;
          if (!mbar_wait(&full[slot], (uint32_t)(q / NS) & 1u)) {
            ok = false;
            break;
          }
          const uint8_t* st = stages + slot * SB;
          const int lo = rb - r0;  // first local row of this stage
          // Quads of local rows owned by this warp that overlap [lo, lo+nr).
          for (int quad = warp; quad * 4 < nrows; quad += DN_CONSUMER_WARPS) {
            const int lr = quad * 4 + sub;
            if (quad * 4 + 3 < lo || quad * 4 >= lo + nr) continue;
            const bool active = lr >= lo && lr < lo + nr && lr < nrows;
            float acc[GROUP_MAX];
#pragma unroll
            for (int m = 0; m < GROUP_MAX; ++m) acc[m] = 0.f;
            if (active) {
              const uint8_t* wrow = st + (size_t)(lr - lo) * row_bytes;
              const uint8_t* srow = nullptr;
              if constexpr (FMT == W_E4M3) {
                const uintptr_t s0 = (uintptr_t)(a.wscale + ((size_t)e * a.H + rb) * (I / 32));
                srow = st + sc_area_off + (s0 & 15) + (size_t)(lr - lo) * (I / 32);
              }
              for (int v = j8; v < nvec; v += 8) Math::step(wrow, srow, v, hrow, cnt, acc);
            }
#pragma unroll
            for (int m = 0; m < GROUP_MAX; ++m) {
              if (m < cnt) {
                float s = acc[m];
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                acc[m] = s;
              }
            }
            if (active && j8 == 0) {
#pragma unroll
              for (int m = 0; m < GROUP_MAX; ++m) {
                if (m < cnt) {
                  float* dst = &acc_tile[tok[m] * a.rows_max + lr];
                  *dst = fmaf(sc[m], acc[m], *dst);
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
        }
      }
      if (!ok && lane == 0) {
        *(volatile int*)&flags[0] = 1;
        raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
      }
    }
    __syncthreads();
    if (flags[0]) return;  // a wait gave up; the status word says so
  }

  // Write this CTA's rows of y for every token.
  for (int i = threadIdx.x; i < a.B * nrows; i += blockDim.x) {
    const int b = i / nrows;
    const int lr = i - b * nrows;
    const float v = acc_tile[b * a.rows_max + lr];
    const size_t o = (size_t)b * a.H + r0 + lr;
    if (a.out_fp32)
      reinterpret_cast<float*>(a.out)[o] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(v);
  }
}

}  // namespace wdb
