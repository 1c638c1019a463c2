// gate_up projection + SiLU on the 5th-generation tensor cores (tcgen05),
// sm_100a.  Same operation and output as moe_gate_up_kernel
// (csrc/moe_gate_up_3d_batched.cu:14-115 of the reference):
//   h[slot, i] = silu(x[tok] . Wgu[e, i, :]) * (x[tok] . Wgu[e, I + i, :]).
//
// Design (B200):
//  * Work item = (expert, tile of 64 neurons).  A group is every routed slot
//    of one expert, so each expert's weights cross HBM once per call.
//  * The A operand is 128 weight rows, gate rows [i0, i0+64) then the
//    matching up rows, fetched by ONE 4-D TMA box over the view
//    (k, neuron, gate|up, expert) of w_gate_up [E, 2I, H]; neurons past I
//    are zero-filled by the TMA unit.  TMEM lane i then holds gate (i < 64)
//    or up (i >= 64) of neuron i0 + (i & 63); the epilogue pairs them
//    through a 2 KB shared-memory exchange.
//  * The B operand is every token of the launch (N = B rounded up to 16,
//    at most 64; rows past B zero-filled), one 2-D TMA box per K stage.
//    The MMA computes all B columns; the epilogue reads only the columns of
//    the group's tokens.  Tensor-core time is far below the weight stream at
//    these N, and x (B x 8 KB) stays in L2.
//  * Warp roles: warp 0 = TMA producer (ring of `stages` stages of `kch`
//    64-wide K chunks: 16 KB of weights + B x 128 B of x per chunk),
//    warp 1 = TMEM allocator + single-thread MMA issuer (4 x K=16 MMAs per
//    64-wide K stage, tcgen05.commit releases the stage), warps 2-5 =
//    epilogue (tcgen05.ld, silu(g) * u, bf16 store).  Two TMEM accumulator
//    buffers let the epilogue of one item overlap the MMAs of the next.
//  * Every wait is bounded; on timeout the CTA raises WD_STATUS_WAIT_TIMEOUT,
//    stops, lets its in-flight copies and MMAs land, frees TMEM and returns.
//  * MXFP8 weights (moe_gate_up_tc_mx_kernel): the producer streams E4M3
//    rows (tiled TMA boxes of 128 K-bytes x the same 128 rows, no swizzle)
//    with their UE8M0 scales into stages of 256 K, and the x chunks of the
//    stage into a ring of their own; eight converter warps (6-13) decode each
//    box into two bf16 K-chunks in the 128-byte-swizzled layout (E4M3 ->
//    bf16 with integer operations, the block scale as one exact power-of-two
//    bf16 multiply) in a ring of converted tiles and free the E4M3 stage as
//    soon as it is decoded, so the weight ring holds bytes in flight rather
//    than bytes waiting for the MMA; the MMA and epilogue are those of the
//    bf16 kernel.
#pragma once

#include "wd_gate_up.cuh"
#include "wd_tc.cuh"

namespace wdb {

constexpr int TC_M = 128;                     // weight rows per tile (64 gate + 64 up)
constexpr int TC_NEUR = 64;                   // neurons per tile
constexpr int TC_BK = 64;                     // K elements per stage (128-byte rows)
constexpr int TC_NMAX = 64;                   // tokens per launch (max MMA N)
constexpr int TC_A_BYTES = TC_M * TC_BK * 2;  // 16 KB
constexpr int TC_THREADS = 6 * 32;
constexpr int TC_MX_CW = 8;                   // converter warps (MXFP8)
constexpr int TC_MX_THREADS = (6 + TC_MX_CW) * 32;
constexpr int TC_MX_NMAX = 16;                // tokens per MXFP8 launch
constexpr int TC_MX_BOX = 128 * 128;          // E4M3 box: 128 rows x 128 K (bytes)
constexpr int TC_MX_SC = 2 * 64 * 16;         // scale box: 128 rows x 16 blocks of 32
constexpr int TC_MX_CONV = 2 * TC_A_BYTES;    // converted box: two bf16 K-chunks
constexpr int TC_MX_STAGE_K = 256;            // K per MXFP8 stage (two E4M3 boxes)
constexpr int TC_TMEM_COLS = 2 * TC_NMAX;     // two fp32 accumulator buffers

struct GateUpTcArgs {
  const int32_t* ids;   // [B, K]
  __nv_bfloat16* out;   // [B*K, I]
  uint32_t* status;
  int B, E, K, H, I;
  int stages;           // smem ring depth
  int npad;             // MMA N: B rounded up to 16 (<= TC_NMAX)
  int kch;              // 64-wide K chunks per stage
  int cl;               // CTAs per cluster: each takes 1/cl of K of every item
  int conv;             // MXFP8: converted-box ring depth (0 for bf16)
  int xstages;          // MXFP8: x ring depth (0 for bf16)
};

constexpr int TC_XCH = 8;                     // members per epilogue exchange round

// One stage: kch A chunks (16 KB each) then kch B chunks (npad rows x 128 B).
__host__ __device__ inline int gate_up_tc_stage_bytes(int kch, int npad) {
  return kch * (TC_A_BYTES + npad * TC_BK * 2);
}

// Split-K partials of one exchange round: [2][cl - 1][TC_XCH members][128 rows].
__host__ __device__ inline int gate_up_tc_xbuf_bytes(int cl) {
  return 2 * (cl - 1) * TC_XCH * TC_M * 4;
}

__host__ inline int gate_up_tc_smem_bytes(int stages, int kch, int npad, int n, int E, int cl) {
  return 1024 + stages * gate_up_tc_stage_bytes(kch, npad) + TC_XCH * TC_NEUR * 4 +
         gate_up_tc_xbuf_bytes(cl) + (2 * stages + 9) * 8 + 16 + CTRL_INTS * 4 +
         route_smem_bytes(n, E, true);
}

// MXFP8 weight stage (256 K): two E4M3 boxes and the scale box of the
// stage's 512-K block (34 KB, a multiple of 1024).  x stage: the stage's four
// 64-wide x chunks (npad rows x 128 B each, 1024-aligned for the swizzle).
constexpr int TC_MX_STAGE = 2 * TC_MX_BOX + TC_MX_SC;
__host__ __device__ inline int gate_up_tc_mx_xstage_bytes(int npad) { return 4 * npad * TC_BK * 2; }

__host__ inline int gate_up_tc_mx_smem_bytes(int stages, int xstages, int conv, int npad, int n,
                                             int E, int cl) {
  return 1024 + stages * TC_MX_STAGE + xstages * gate_up_tc_mx_xstage_bytes(npad) +
         conv * TC_MX_CONV + TC_XCH * TC_NEUR * 4 + gate_up_tc_xbuf_bytes(cl) +
         (2 * stages + 9 + 2 * conv + 2 * xstages) * 8 + 16 + CTRL_INTS * 4 +
         route_smem_bytes(n, E, true);
}

// Sixteen E4M3 bytes of one row (one 32-element block half) -> sixteen bf16
// weights times the block scale 2^(s - 127), exact: e4m3x16_to_bf16 gives the
// values times 2^-120, so the factor is 2^(s - 7), one bf16 multiply while
// it is a bf16 normal (s <= 134), two above.  A NaN byte or scale byte 255
// makes all sixteen NaN (so is every output that uses them, as with the
// dequantised weights).
__device__ __forceinline__ void mx_decode_scaled(const uint4& v, uint32_t s, uint32_t (&p)[8]) {
  const bool nan_byte = e4m3x16_to_bf16(v, p);
  uint32_t m1 = (s + 120u) << 7, m2 = 0u;
  if (nan_byte || s == 255u) {
    m1 = 0x7fc0u;
  } else if (s > 134u) {
    m1 = 0x7f00u;              // 2^127
    m2 = (s - 7u) << 7;        // 2^(s - 134)
  }
  const __nv_bfloat162 f1 = __halves2bfloat162(__ushort_as_bfloat16((unsigned short)m1),
                                               __ushort_as_bfloat16((unsigned short)m1));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&p[i]);
    b = __hmul2(b, f1);
    p[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  if (m2) {
    const __nv_bfloat162 f2 = __halves2bfloat162(__ushort_as_bfloat16((unsigned short)m2),
                                                 __ushort_as_bfloat16((unsigned short)m2));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&p[i]);
      b = __hmul2(b, f2);
      p[i] = *reinterpret_cast<uint32_t*>(&b);
    }
  }
}

// One E4M3 box (128 rows x 128 K-bytes, rows 128 B apart, at src) -> two
// bf16 K-chunks of the 128-byte-swizzled K-major layout at dst and dst +
// 16 KB, run by all TC_MX_CW converter warps (cw = converter warp index).
// The scale byte of (row, 16-byte unit c16) is sc[row * sc_row + (c16 >> 1)]
// (sc already offset to the box's first 32-element block).
//
// Per box, warp cw and unit u < 4 cover rows 32u + 4cw .. +3, all eight
// 16-byte K units (c16) of each row.  16-byte shared accesses are served per
// quarter warp (8 lanes), so each quarter must touch 8 different 16-byte bank
// groups: quarter q = 2 pair + half takes units 0-3 of row 2 pair + half and
// units 4-7 of row 2 pair + (half ^ 1).  The loads then hit groups c16, and
// the bf16 stores (swizzled unit (2 (c16 & 3) + t) ^ (row & 7), t = 0, 1)
// hit two disjoint sets of four because the two rows differ in bit 0.  The
// four units are independent (loads first, then decode and stores), so the
// decode's integer chains overlap.
__device__ __forceinline__ void mx_convert_box(const uint8_t* src, uint8_t* dst,
                                               const uint8_t* sc, int sc_row, int cw, int lane) {
  constexpr int NU = TC_M / (4 * TC_MX_CW);  // units per thread per box
  const int c16 = lane & 7;
  const int rsub = 2 * ((lane >> 4) & 1) + (((lane >> 2) & 1) ^ ((lane >> 3) & 1));
  uint4 v[NU];
  uint32_t sbyte[NU];
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int row = 4 * TC_MX_CW * u + 4 * cw + rsub;
    v[u] = lds16(src + row * 128 + c16 * 16);
    sbyte[u] = sc[row * sc_row + (c16 >> 1)];
  }
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int row = 4 * TC_MX_CW * u + 4 * cw + rsub;
    uint32_t p[8];
    mx_decode_scaled(v[u], sbyte[u], p);
    uint8_t* drow = dst + (c16 >> 2) * TC_A_BYTES + row * 128;
    const int u0 = (c16 & 3) * 2;
    *reinterpret_cast<uint4*>(drow + ((u0 ^ (row & 7)) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
    *reinterpret_cast<uint4*>(drow + (((u0 + 1) ^ (row & 7)) << 4)) =
        make_uint4(p[4], p[5], p[6], p[7]);
  }
}

// Body of both kernels.  kMx: MXFP8 weights (tm_w over E4M3 bytes, tm_s over
// the scales, converter warps); else bf16 weights.  kRoute: routing code
// compiled for this launch's slot count (RouteMode).
// kFused: phase 1 of moe_ffn_tc_kernel (FusedCtx: shared-memory region,
// routing and TMEM given; the barriers are invalidated at the end so that the
// down phase can reuse the memory).
template <bool kMx, int kRoute, bool kFused = false>
__device__ __forceinline__ void gate_up_tc_body(const CUtensorMap& tm_w, const CUtensorMap& tm_x,
                                                const CUtensorMap* tm_s, const GateUpTcArgs a,
                                                const FusedCtx* fx = nullptr) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = kFused ? fx->base : smem_raw + pad;
  const int S = a.stages;
  const int KCH = a.kch;
  const int BT = a.npad * TC_BK * 2;  // bytes of one B chunk
  const int SB = kMx ? TC_MX_STAGE : gate_up_tc_stage_bytes(KCH, a.npad);
  const int CL = a.cl;
  const int CS = kMx ? a.conv : 0;
  const int SX = kMx ? a.xstages : 0;
  const int XB = kMx ? gate_up_tc_mx_xstage_bytes(a.npad) : 0;
  uint8_t* ring = base;
  uint8_t* xring = ring + (size_t)S * SB;  // MXFP8: [SX] x stages
  uint8_t* conv = xring + (size_t)SX * XB;  // MXFP8: [CS] converted boxes (2 bf16 K-chunks)
  float* xch = reinterpret_cast<float*>(conv + (size_t)CS * TC_MX_CONV);  // [TC_XCH][64]
  float* xbuf = xch + TC_XCH * TC_NEUR;  // [2][CL-1][TC_XCH][128] (cluster rank 0)
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xbuf) +
                                               gate_up_tc_xbuf_bytes(CL));
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2] accumulator ready
  uint64_t* tempty = tfull + 2;  // [2] accumulator drained
  uint64_t* done = tempty + 2;   // MMA drain
  uint64_t* xfull = done + 1;    // [2] rank 0: partials of a round arrived
  uint64_t* xempty = xfull + 2;  // [2] ranks > 0: rank 0 consumed a round's slot
  uint64_t* cfull = xempty + 2;  // MXFP8: [CS] converted box written
  uint64_t* cempty = cfull + CS; // MXFP8: [CS] converted box read by the MMAs
  uint64_t* bfull = cempty + CS; // MXFP8: [SX] x stage landed
  uint64_t* bempty = bfull + SX; // MXFP8: [SX] x stage read by the MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bempty + SX);
  volatile int* ctrl = reinterpret_cast<volatile int*>(tmem_slot + 4);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;

  const int n = a.B * a.K;
  const RouteSmem r = kFused ? *fx->r : route_carve(route_base, n, a.E, true);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Barrier set-up and the TMEM allocation overlap the topk_ids loads.
  auto setup = [&]() {
    if (threadIdx.x == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], kMx ? TC_MX_CW : 1);  // MXFP8: freed by the converter warps
      }
      mbar_init(&tfull[0], 1);
      mbar_init(&tfull[1], 1);
      mbar_init(&tempty[0], 4);
      mbar_init(&tempty[1], 4);
      mbar_init(done, 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&xfull[b], (uint32_t)max(1, CL - 1) * 128u);
        mbar_init(&xempty[b], 128u);
      }
      for (int c = 0; c < CS; ++c) {
        mbar_init(&cfull[c], TC_MX_CW);  // one arrival per converter warp
        mbar_init(&cempty[c], 1);
      }
      for (int c = 0; c < SX; ++c) {
        mbar_init(&bfull[c], 1);
        mbar_init(&bempty[c], 1);
      }
      ctrl[0] = 0;
      fence_mbar_init();
    }
    if (threadIdx.x == 32) {
      prefetch_tensormap(&tm_w);
      prefetch_tensormap(&tm_x);
      if (kMx) prefetch_tensormap(tm_s);
    }
    if (!kFused && warp == 1) {
      tmem_alloc(tmem_slot, TC_TMEM_COLS);
      tmem_relinquish();
      tc_fence_before();
    }
  };
  if constexpr (kFused) {
    setup();
    __syncthreads();
  } else {
    route_build<false, decltype(setup), kRoute>(r, a.ids, n, a.E, a.K, true, MAX_SLOTS, a.status,
                                               setup);  // ends with __syncthreads
  }
  tc_fence_after();
  const uint32_t tmem = kFused ? fx->tmem : *tmem_slot;

  const int n_tiles = (a.I + TC_NEUR - 1) / TC_NEUR;
  const int items = *r.nsg * n_tiles;
  // K units of a row: 64-wide chunks (bf16) or 256-wide stages (MXFP8).
  const int nkc_all = kMx ? (a.H + TC_MX_STAGE_K - 1) / TC_MX_STAGE_K : (a.H + TC_BK - 1) / TC_BK;
  // Cluster rank `crank` of cluster `cid` covers units [kc_lo, kc_lo + nkc)
  // of every item of its cluster; rank 0 sums the partials and stores h.
  const int crank = CL > 1 ? (int)cluster_ctarank() : 0;
  const int kc_lo = crank * nkc_all / CL;
  const int nkc = (crank + 1) * nkc_all / CL - kc_lo;
  const int nk = kMx ? nkc : (nkc + KCH - 1) / KCH;  // stages per item
  const int G = (int)gridDim.x / CL;           // clusters
  const int cid = (int)blockIdx.x / CL;

  // Bounded wait that also gives up once another role has aborted.
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
    // ---------------- TMA producer ----------------
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    uint32_t it = 0;
    uint32_t nwi = 0, nx = 0;  // MXFP8: weight stages and x stages issued
    bool ok = true;
    for (int t = cid; ok && t < items; t += G) {
      const int g = t / n_tiles, mt = t - g * n_tiles;
      const int e = r.sg_exp[g];
      if (e < 0) continue;
      for (int ks = 0; ks < nk; ++ks, ++it) {
        const int slot = (int)(it % (uint32_t)S);
        const uint32_t ph = (it / (uint32_t)S) & 1u;
        if (lane == 0) {
          if (!wait(&empty[slot], ph ^ 1u)) {
            ok = false;
          } else if constexpr (kMx) {
            // The two E4M3 boxes and the scales of the 512-K block (every
            // box in bounds: the host requires hidden % 512 == 0), then the
            // stage's x chunks into the x ring.
            const int k0 = (kc_lo + ks) * TC_MX_STAGE_K;
            uint8_t* w8 = ring + (size_t)slot * SB;
            mbar_arrive_expect_tx(&full[slot], (uint32_t)SB);
            for (int j = 0; j < 2; ++j)
              tma_load_4d(w8 + j * TC_MX_BOX, &tm_w, k0 + j * 128, mt * TC_NEUR, 0, e, &full[slot],
                          pol_w);
            tma_load_4d(w8 + 2 * TC_MX_BOX, tm_s, (k0 >> 9) * 16, mt * TC_NEUR, 0, e, &full[slot],
                        pol_w);
            nwi = it + 1;
            const int xs = (int)(it % (uint32_t)SX);
            if (!wait(&bempty[xs], ((it / (uint32_t)SX) & 1u) ^ 1u)) {
              ok = false;
            } else {
              uint8_t* xst = xring + (size_t)xs * XB;
              mbar_arrive_expect_tx(&bfull[xs], (uint32_t)XB);
              for (int c = 0; c < 4; ++c)
                tma_load_2d(xst + c * BT, &tm_x, k0 + c * TC_BK, 0, &bfull[xs], pol_x);
              nx = it + 1;
            }
          } else {
            const int c0 = kc_lo + ks * KCH, nc = min(KCH, kc_lo + nkc - c0);
            uint8_t* st = ring + (size_t)slot * SB;
            mbar_arrive_expect_tx(&full[slot], (uint32_t)nc * (TC_A_BYTES + BT));
            for (int c = 0; c < nc; ++c)
              tma_load_4d(st + c * TC_A_BYTES, &tm_w, (c0 + c) * TC_BK, mt * TC_NEUR, 0, e,
                          &full[slot], pol_w);
            for (int c = 0; c < nc; ++c)
              tma_load_2d(st + KCH * TC_A_BYTES + c * BT, &tm_x, (c0 + c) * TC_BK, 0, &full[slot],
                          pol_x);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
    }
    // After an abort let every issued copy land before the CTA can exit
    // (MXFP8: the weight stage `it` may be in flight while its x stage is not).
    if (!ok && lane == 0) {
      const uint32_t nw = kMx ? nwi : it;
      const uint32_t lo = nw > (uint32_t)S ? nw - (uint32_t)S : 0u;
      for (uint32_t i = lo; i < nw; ++i) {
        uint64_t* bar = &full[i % (uint32_t)S];
        const uint32_t ph = (i / (uint32_t)S) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar, ph) && globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
        }
      }
      if constexpr (kMx) {
        const uint32_t xlo = nx > (uint32_t)SX ? nx - (uint32_t)SX : 0u;
        for (uint32_t i = xlo; i < nx; ++i) {
          uint64_t* bar = &bfull[i % (uint32_t)SX];
          const uint32_t ph = (i / (uint32_t)SX) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(bar, ph) && globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread) ----------------
    if (lane == 0) {
      uint32_t it = 0, vi = 0, ci = 0;
      bool ok = true;
      bool issued = false;
      for (int t = cid; ok && t < items; t += G) {
        const int g = t / n_tiles;
        if (r.sg_exp[g] < 0) continue;
        const uint32_t buf = vi & 1u;
        if (!wait(&tempty[buf], ((vi >> 1) & 1u) ^ 1u)) { ok = false; break; }
        tc_fence_after();
        const uint32_t idesc = tc_idesc_bf16(TC_M, a.npad);
        const uint32_t d = tmem + buf * TC_NMAX;
        for (int ks = 0; ks < nk; ++ks, ++it) {
          const int slot = (int)(it % (uint32_t)S);
          if constexpr (kMx) {
            // Box j of the stage, once converted: K-chunks 2j, 2j + 1 (A from
            // the converted ring, B = the stage's x chunks in the x ring).
            const int xs = (int)(it % (uint32_t)SX);
            if (!wait(&bfull[xs], (it / (uint32_t)SX) & 1u)) { ok = false; break; }
            tc_fence_after();
            const uint8_t* st = xring + (size_t)xs * XB;
            for (int j = 0; j < 2; ++j, ++ci) {
              const int cs = (int)(ci % (uint32_t)CS);
              if (!wait(&cfull[cs], (ci / (uint32_t)CS) & 1u)) { ok = false; break; }
              tc_fence_after();
              for (int hh = 0; hh < 2; ++hh) {
                const uint64_t ad =
                    tc_desc_sw128(smem_u32(conv + (size_t)cs * TC_MX_CONV + hh * TC_A_BYTES));
                const uint64_t bd = tc_desc_sw128(smem_u32(st + (2 * j + hh) * BT));
#pragma unroll
                for (int kk = 0; kk < TC_BK / 16; ++kk)
                  tc_mma_bf16(d, ad + 2u * kk, bd + 2u * kk, idesc,
                              (ks | j | hh | kk) != 0 ? 1u : 0u);
              }
              tc_commit(&cempty[cs]);
              issued = true;
            }
            if (!ok) break;
            tc_commit(&bempty[xs]);
          } else {
            if (!wait(&full[slot], (it / (uint32_t)S) & 1u)) { ok = false; break; }
            tc_fence_after();
            const uint8_t* st = ring + (size_t)slot * SB;
            const int nc = min(KCH, nkc - ks * KCH);
            for (int c = 0; c < nc; ++c) {
              const uint64_t ad = tc_desc_sw128(smem_u32(st + c * TC_A_BYTES));
              const uint64_t bd = tc_desc_sw128(smem_u32(st + KCH * TC_A_BYTES + c * BT));
#pragma unroll
              for (int kk = 0; kk < TC_BK / 16; ++kk)
                tc_mma_bf16(d, ad + 2u * kk, bd + 2u * kk, idesc, (ks | c | kk) != 0 ? 1u : 0u);
            }
            tc_commit(&empty[slot]);
            issued = true;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[buf]);
        ++vi;
      }
      // Every MMA this thread issued has completed before TMEM is freed.
      if (issued) {
        tc_commit(done);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(done, 0) && globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
        }
      }
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ---------------- MXFP8 converters: warps 6..13 (mx_convert_box) -----
    if constexpr (kMx) {
    const int cw = warp - 6;
    uint32_t it = 0, ci = 0;
    bool ok = true;
    for (int t = cid; ok && t < items; t += G) {
      if (r.sg_exp[t / n_tiles] < 0) continue;
      for (int ks = 0; ks < nk; ++ks, ++it) {
        const int slot = (int)(it % (uint32_t)S);
        if (!wait(&full[slot], (it / (uint32_t)S) & 1u)) { ok = false; break; }
        const uint8_t* w8 = ring + (size_t)slot * SB;
        const uint8_t* sc = w8 + 2 * TC_MX_BOX;
        // first scale block of this stage within the 512-K scale box
        const int sb0 = (((kc_lo + ks) * TC_MX_STAGE_K) & 511) >> 5;
        for (int j = 0; j < 2; ++j, ++ci) {
          const int cs = (int)(ci % (uint32_t)CS);
          if (!wait(&cempty[cs], ((ci / (uint32_t)CS) & 1u) ^ 1u)) { ok = false; break; }
          // box j starts at scale block sb0 + 4 j of the 16-byte scale rows
          mx_convert_box(w8 + j * TC_MX_BOX, conv + (size_t)cs * TC_MX_CONV, sc + sb0 + j * 4, 16,
                         cw, lane);
          fence_proxy_async_smem();  // generic writes -> tensor-core reads
          __syncwarp();
          if (lane == 0) mbar_arrive(&cfull[cs]);
        }
        if (!ok) break;
        // Both boxes decoded: the E4M3 stage goes back to the producer.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }
    }
  } else {
    // ---------------- epilogue: warps 2..5, TMEM lane quarter warp % 4 -----
    // Quarters 0, 1 read gate rows (neurons 32q + lane), quarters 2, 3 the
    // up rows of the same neurons; up values cross over in `xch`.  With
    // clusters (CL > 1) ranks > 0 push their FP32 partials of each round of
    // TC_XCH members into rank 0's `xbuf` over distributed shared memory;
    // rank 0 adds them in rank order and alone stores h.
    const int q = warp & 3;
    const bool is_gate = q < 2;
    const int I = a.I;
    const int row = 32 * q + lane;  // TMEM lane = A row
    uint32_t vi = 0, rr = 0;        // valid items, exchange rounds
    auto waitc = [&](uint64_t* bar, uint32_t parity) -> bool {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 31u) == 31u && ctrl[0]) return false;
        if ((it & 31u) == 31u && globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) {
          raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
          ctrl[0] = 1;
          return false;
        }
      }
    };
    for (int t = cid; t < items; t += G) {
      const int g = t / n_tiles, mt = t - g * n_tiles;
      const int e = r.sg_exp[g];
      const int cnt = r.sg_cnt[g], beg = r.sg_beg[g];
      const int nn = mt * TC_NEUR + 32 * (q & 1) + lane;
      if (e < 0) {
        // A slot with an out-of-range expert id yields zeros.
        if (crank == 0 && is_gate && nn < I)
          for (int c = 0; c < cnt; ++c)
            a.out[(size_t)r.members[beg + c] * I + nn] = __float2bfloat16_rn(0.f);
        continue;
      }
      const uint32_t buf = vi & 1u;
      // A failed (timed-out) wait still runs the exchange rounds so the four
      // warps meet at every bar.sync; nothing is stored from such an item.
      bool got = wait(&tfull[buf], (vi >> 1) & 1u);
      __syncwarp();  // tcgen05.ld and bar.sync below are warp-collective
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + buf * TC_NMAX;
      for (int c0 = 0; c0 < cnt; c0 += TC_XCH, ++rr) {
        // Column of member c = its token; members past cnt re-read column 0.
        float v[TC_XCH];
#pragma unroll
        for (int j = 0; j < TC_XCH; ++j) {
          const int tok = c0 + j < cnt ? r.mtok[beg + c0 + j] : 0;
          v[j] = __uint_as_float(tmem_ld_x1(taddr + (uint32_t)tok));
        }
        tmem_wait_ld();
        if (CL > 1) {
          const uint32_t xb = rr & 1u, xpar = (rr >> 1) & 1u;
          float* slot0 = xbuf + (size_t)xb * (CL - 1) * TC_XCH * TC_M;
          if (crank > 0) {
            // Wait until rank 0 has consumed this slot's previous round, push
            // this rank's partials, signal rank 0.
            got = waitc(&xempty[xb], xpar ^ 1u) && got;
            float* dst = slot0 + (size_t)(crank - 1) * TC_XCH * TC_M + row;
#pragma unroll
            for (int j = 0; j < TC_XCH; ++j) dsmem_st_f32(dsmem_addr(dst + j * TC_M, 0), v[j]);
            mbar_arrive_remote(dsmem_addr(&xfull[xb], 0));
            continue;  // ranks > 0 store nothing
          }
          got = waitc(&xfull[xb], xpar) && got;
          for (int k = 1; k < CL; ++k) {
            const float* src = slot0 + (size_t)(k - 1) * TC_XCH * TC_M + row;
#pragma unroll
            for (int j = 0; j < TC_XCH; ++j) v[j] += src[j * TC_M];
          }
          for (int k = 1; k < CL; ++k) mbar_arrive_remote(dsmem_addr(&xempty[xb], (uint32_t)k));
        }
        if (!is_gate) {
#pragma unroll
          for (int j = 0; j < TC_XCH; ++j) xch[j * TC_NEUR + 32 * (q & 1) + lane] = v[j];
        }
        named_barrier_sync(1, 128);
        if (is_gate && got && nn < I) {
#pragma unroll
          for (int j = 0; j < TC_XCH; ++j) {
            if (c0 + j < cnt) {
              const float u = xch[j * TC_NEUR + 32 * q + lane];
              a.out[(size_t)r.members[beg + c0 + j] * I + nn] =
                  __float2bfloat16_rn(silu_f32(v[j]) * u);
            }
          }
        }
        named_barrier_sync(1, 128);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      ++vi;
    }
  }

  tc_fence_before();
  __syncthreads();
  // h of this CTA is stored: a following down kernel launched with
  // programmatic dependence may start once every CTA got here (as in
  // moe_gate_up_kernel; it waits for this grid before reading h).
  if (!kFused && threadIdx.x == 0) pdl_launch_dependents();
  if (!kFused && warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TC_TMEM_COLS);
  }
  // No CTA leaves while a peer may still write into its shared memory.
  if (CL > 1) cluster_sync();
  if constexpr (kFused) {
    // Every wait and every arrive (local or from the cluster) is done.  This
    // thread's generic shared-memory writes (the epilogue's exchange) are
    // ordered before the down phase's bulk copies into the same bytes.
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
      for (int i = 0; i < 2 * S + 9 + 2 * CS + 2 * SX; ++i) mbar_inval(full + i);
    }
    __syncthreads();
  }
}

template <int kRoute>
__global__ void __launch_bounds__(TC_THREADS, 1)
    moe_gate_up_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_x, const GateUpTcArgs a) {
  gate_up_tc_body<false, kRoute>(tm_w, tm_x, nullptr, a);
}

// MXFP8 weights: tm_w over the E4M3 bytes [E, 2I, H], tm_s over the UE8M0
// scales [E, 2I, H / 32], both viewed as (k, neuron, gate|up, expert).
template <int kRoute>
__global__ void __launch_bounds__(TC_MX_THREADS, 1)
    moe_gate_up_tc_mx_kernel(const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ CUtensorMap tm_x,
                             const __grid_constant__ CUtensorMap tm_s, const GateUpTcArgs a) {
  gate_up_tc_body<true, kRoute>(tm_w, tm_x, &tm_s, a);
}

}  // namespace wdb
