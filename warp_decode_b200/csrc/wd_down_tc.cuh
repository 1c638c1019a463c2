// down projection + top-k weighted sum on the tcgen05 tensor cores, sm_100a.
// Same operation and output as moe_down_kernel
// (csrc/moe_down_3d_batched.cu:45-122 of the reference):
//   y[b, j] = sum_s topk_scale[b,s] * (h[b*topk+s, :] . Wd[e_s, j, :]).
//
// Design (B200):
//  * CTA c owns output rows [c*R, (c+1)*R) of every token (R = 16..64, the
//    MMA N), so the top-k sum never leaves the CTA: no atomics, no scratch.
//  * Operands are swapped relative to a GEMM over weights: per expert group
//    (every routed slot of one expert, at most 128), A = the members' h rows
//    (M = 128, K = inter) gathered from global memory by the worker warps
//    into the 128-byte-swizzled K-major layout, B = the expert's R weight
//    rows (N = R, K = inter), one 3-D TMA box per 64-wide K chunk.  D[m, j]
//    (TMEM lane m, column j) is member m's dot product for row j.
//  * Each expert's R x inter weight block (12 KB at R = 32, inter = 192) is
//    one ring stage; every CTA walks all touched experts in the same order.
//  * Worker warps (2-5): gather A for item i, then drain D of item i-1:
//    thread m adds topk_scale * D[m, :] into an FP32 tile Y[token][R] in
//    shared memory (repeated tokens inside a group in separate rounds, so
//    the summation order is fixed: deterministic).  At the end Y -> y.
//  * Warp 0 = weight TMA producer, warp 1 = TMEM allocator + MMA issuer.
//    A and D are double-buffered.  Every wait is bounded (status bit on
//    timeout).
#pragma once

#include "wd_down.cuh"
#include "wd_tc.cuh"

namespace wdb {

constexpr int DTC_M = 128;              // member rows per MMA (A rows)
constexpr int DTC_BK = 64;              // K elements per chunk (128-byte rows)
constexpr int DTC_MAXKC = 4;            // inter <= 256
constexpr int DTC_THREADS = 6 * 32;
constexpr int DTC_A_CHUNK = DTC_M * DTC_BK * 2;  // 16 KB

struct DownTcArgs {
  const __nv_bfloat16* h;  // [B*K, I]
  const int32_t* ids;      // [B, K]
  const float* scale;      // [B, K]
  void* out;               // [B, H] bf16 or fp32
  int out_fp32;
  uint32_t* status;
  int B, E, K, H, I;
  int R;                   // rows per CTA (MMA N)
  int stages;
};

__host__ __device__ inline int down_tc_stage_bytes(int R, int I) {
  return ((I + DTC_BK - 1) / DTC_BK) * R * DTC_BK * 2;
}

__host__ inline int down_tc_smem_bytes(int stages, int R, int I, int B, int n, int E) {
  const int kc = (I + DTC_BK - 1) / DTC_BK;
  return 1024 + 2 * kc * DTC_A_CHUNK + stages * down_tc_stage_bytes(R, I) +
         ((B * (R + 1) * 4 + 127) / 128) * 128 + ((n * 4 + 127) / 128) * 128 * 2 +
         (2 * stages + 9) * 8 + 16 + CTRL_INTS * 4 + route_smem_bytes(n, E, true);
}

// D row of this thread's lane: R consecutive fp32 columns.
template <int R>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float (&v)[R]) {
#pragma unroll
  for (int c = 0; c < R; c += 8) {
    uint32_t u[8];
    tmem_ld_x8(taddr + (uint32_t)c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[c + j] = __uint_as_float(u[j]);
  }
}

template <int R>
__global__ void __launch_bounds__(DTC_THREADS, 1)
    moe_down_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const DownTcArgs a) {
  static_assert(R == 16 || R == 32 || R == 64, "rows per CTA");
  constexpr uint32_t DTC_TMEM_COLS = 2 * R < 32 ? 32 : 2 * R;  // two D buffers
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = smem_raw + pad;
  const int S = a.stages;
  const int I = a.I;
  const int kc = (I + DTC_BK - 1) / DTC_BK;
  const int n = a.B * a.K;
  const int SB = down_tc_stage_bytes(R, I);
  const int WCH = R * DTC_BK * 2;  // bytes of one weight chunk
  uint8_t* abuf = base;                                   // [2][kc][128 x 128 B]
  uint8_t* ring = abuf + 2 * (size_t)kc * DTC_A_CHUNK;    // [S][kc][R x 128 B]
  float* Y = reinterpret_cast<float*>(ring + (size_t)S * SB);  // [B][R + 1]
  float* s_scale = Y + ((a.B * (R + 1) * 4 + 127) / 128) * 32;
  int* s_rank = reinterpret_cast<int*>(s_scale + ((n * 4 + 127) / 128) * 32);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(s_rank + ((n * 4 + 127) / 128) * 32);
  uint64_t* wempty = wfull + S;
  uint64_t* afull = wempty + S;   // [2]
  uint64_t* aempty = afull + 2;   // [2]
  uint64_t* dfull = aempty + 2;   // [2]
  uint64_t* dempty = dfull + 2;   // [2]
  uint64_t* done = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* ctrl = reinterpret_cast<volatile int*>(tmem_slot + 4);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;
  const RouteSmem r = route_carve(route_base, n, a.E, true);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int j0 = (int)blockIdx.x * R;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 4);
      mbar_init(&aempty[b], 1);
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 4);
    }
    mbar_init(done, 1);
    ctrl[0] = 0;
    fence_mbar_init();
  }
  if (threadIdx.x == 32) prefetch_tensormap(&tm_w);
  if (warp == 1) {
    tmem_alloc(tmem_slot, DTC_TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  // h, topk_scale (and possibly topk_ids) come from the preceding kernel.
  pdl_wait_primary();
  route_build(r, a.ids, n, a.E, a.K, true, DTC_M, a.status);  // ends with __syncthreads
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_scale[i] = a.scale[i];
  // Rank of each member among earlier members of its group with the same
  // token (members are in slot order, so repeats of a token are adjacent),
  // and per group the largest rank (kept in r.aux).
  const int nsg = *r.nsg;
  for (int g = threadIdx.x; g < nsg; g += blockDim.x) {
    const int b = r.sg_beg[g], c = r.sg_cnt[g];
    int rk = 0, mx = 0;
    for (int p = 0; p < c; ++p) {
      rk = (p > 0 && r.mtok[b + p] == r.mtok[b + p - 1]) ? rk + 1 : 0;
      s_rank[b + p] = rk;
      mx = max(mx, rk);
    }
    r.aux[g] = mx;
  }
  for (int i = threadIdx.x; i < a.B * (R + 1); i += blockDim.x) Y[i] = 0.f;
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (mbar_try_wait(bar, parity)) return true;
      if ((it & 31u) == 0) {
        if (ctrl[0]) return false;
        if (globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) {
          raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
          ctrl[0] = 1;
          return false;
        }
      }
    }
  };

  if (warp == 0) {
    // ---------------- weight producer ----------------
    const uint64_t pol = l2_policy_evict_first();
    uint32_t it = 0;
    bool ok = true;
    for (int g = 0; ok && g < nsg; ++g) {
      const int e = r.sg_exp[g];
      if (e < 0) continue;
      const int slot = (int)(it % (uint32_t)S);
      if (lane == 0) {
        if (!wait(&wempty[slot], ((it / (uint32_t)S) & 1u) ^ 1u)) {
          ok = false;
        } else {
          uint8_t* st = ring + (size_t)slot * SB;
          mbar_arrive_expect_tx(&wfull[slot], (uint32_t)(kc * WCH));
          for (int c = 0; c < kc; ++c)
            tma_load_3d(st + c * WCH, &tm_w, c * DTC_BK, j0, e, &wfull[slot], pol);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) ++it;
    }
    if (!ok && lane == 0) {
      const uint32_t lo = it > (uint32_t)S ? it - (uint32_t)S : 0u;
      for (uint32_t i = lo; i < it; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&wfull[i % (uint32_t)S], (i / (uint32_t)S) & 1u) &&
               globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true, issued = false;
      const uint32_t idesc = tc_idesc_bf16(DTC_M, R);
      for (int g = 0; ok && g < nsg; ++g) {
        if (r.sg_exp[g] < 0) continue;
        const uint32_t b = it & 1u, ph2 = (it >> 1) & 1u;
        const int slot = (int)(it % (uint32_t)S);
        if (!wait(&afull[b], ph2) || !wait(&dempty[b], ph2 ^ 1u) ||
            !wait(&wfull[slot], (it / (uint32_t)S) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* A = abuf + (size_t)b * kc * DTC_A_CHUNK;
        const uint8_t* W = ring + (size_t)slot * SB;
        const uint32_t d = tmem + b * R;
        for (int c = 0; c < kc; ++c) {
          const uint64_t ad = tc_desc_sw128(smem_u32(A + c * DTC_A_CHUNK));
          const uint64_t bd = tc_desc_sw128(smem_u32(W + c * WCH));
#pragma unroll
          for (int kk = 0; kk < DTC_BK / 16; ++kk)
            tc_mma_bf16(d, ad + 2u * kk, bd + 2u * kk, idesc, (c | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&wempty[slot]);
        tc_commit(&aempty[b]);
        tc_commit(&dfull[b]);
        issued = true;
        ++it;
      }
      if (issued) {
        tc_commit(done);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(done, 0) && globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- workers: gather A (item i), drain D (item i-1) ----
    const int wt = threadIdx.x - 64;  // 0..127
    const int q = warp & 3;           // TMEM lane quarter
    const int vecs = I / 8;           // 16-byte pieces per h row
    int prev_g = -1;
    uint32_t it = 0;
    auto drain = [&](int g, uint32_t j) {
      const uint32_t b = j & 1u;
      const bool got = wait(&dfull[b], (j >> 1) & 1u);
      __syncwarp();  // tcgen05.ld and bar.sync below are warp-collective
      tc_fence_after();
      const int beg = r.sg_beg[g], cnt = r.sg_cnt[g], mr = r.aux[g];
      const int m = 32 * q + lane;
      float v[R];
      if (32 * q < cnt) {  // warp-uniform: this quarter holds members
        tmem_ld_row<R>(tmem + ((uint32_t)(32 * q) << 16) + b * R, v);
        tmem_wait_ld();
      }
      const bool act = got && m < cnt;
      const int rk_m = act ? s_rank[beg + m] : -1;
      float* yrow = Y + (act ? r.mtok[beg + m] : 0) * (R + 1);
      const float sc = act ? s_scale[r.members[beg + m]] : 0.f;
      // Round rk adds the members that are the rk-th slot of their token in
      // this group; every thread runs every round (bar.sync stays convergent).
      for (int rk = 0; rk <= mr; ++rk) {
        if (rk_m == rk) {
#pragma unroll
          for (int jj = 0; jj < R; ++jj) yrow[jj] = fmaf(sc, v[jj], yrow[jj]);
        }
        if (mr > 0) named_barrier_sync(1, 128);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[b]);
    };
    for (int g = 0; g < nsg; ++g) {
      if (r.sg_exp[g] < 0) continue;  // invalid ids contribute nothing
      const uint32_t b = it & 1u;
      const bool got = wait(&aempty[b], ((it >> 1) & 1u) ^ 1u);
      const int beg = r.sg_beg[g], cnt = r.sg_cnt[g];
      uint8_t* A = abuf + (size_t)b * kc * DTC_A_CHUNK;
      if (got) {
        for (int pc = wt; pc < cnt * kc * 8; pc += 128) {
          const int p = pc / (kc * 8), rem = pc - p * (kc * 8);
          const int c = rem >> 3, j = rem & 7;
          const int kv = c * 8 + j;  // 16-byte piece of the row
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (kv < vecs) v = ldg16(a.h + (size_t)r.members[beg + p] * I + kv * 8);
          *reinterpret_cast<uint4*>(A + c * DTC_A_CHUNK + (p >> 3) * 1024 + (p & 7) * 128 +
                                    ((j ^ (p & 7)) << 4)) = v;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[b]);
      if (prev_g >= 0) drain(prev_g, it - 1);
      prev_g = g;
      ++it;
    }
    if (prev_g >= 0) drain(prev_g, it - 1);
    named_barrier_sync(1, 128);
    // Y -> y rows [j0, j0 + R) of every token.
    for (int i = wt; i < a.B * R; i += 128) {
      const int t = i / R, jj = i - t * R;
      if (j0 + jj < a.H) {
        const float v = Y[t * (R + 1) + jj];
        if (a.out_fp32)
          reinterpret_cast<float*>(a.out)[(size_t)t * a.H + j0 + jj] = v;
        else
          reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.H + j0 + jj] =
              __float2bfloat16_rn(v);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, DTC_TMEM_COLS);
  }
}

}  // namespace wdb
