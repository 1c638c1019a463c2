// down projection + top-k weighted sum on the tcgen05 tensor cores, sm_100a.
// Same operation and output as moe_down_kernel
// (csrc/moe_down_3d_batched.cu:45-122 of the reference):
//   y[b, j] = sum_s topk_scale[b,s] * (h[b*topk+s, :] . Wd[e_s, j, :]).
//
// Design (B200):
//  * A cluster of CL CTAs owns a tile of 128 output rows for every token;
//    the CTAs of the cluster split the touched experts between them (group
//    g goes to cluster rank g % CL) and at the end sum their FP32 partial
//    tiles through distributed shared memory in a fixed rank order.  The
//    top-k sum never leaves the cluster: no atomics, no global scratch,
//    deterministic.
//  * Per item (one expert, at most DTC_N of its routed slots):
//      A = the expert's 128 weight rows of the tile (M = 128, K = inter),
//          one 3-D TMA box per 64-wide K chunk (16 KB each), up to 4
//          chunks per ring stage (inter up to 2048: several stages);
//      B = the members' h rows (N = 16), gathered by the gather warps into
//          the 128-byte-swizzled K-major layout one weight stage's K range
//          at a time (h slices: shared memory no longer grows with inter);
//      D[j, c] (TMEM lane j, column c) = row j . h[member c].
//  * Epilogue warps add topk_scale[c] * D[j, c] into Y[token(c)][j] in
//    shared memory, one thread per row, members in slot order (so repeated
//    tokens add in a fixed order).
//  * Warp roles: 0 = weight TMA producer, 1 = TMEM allocator + MMA issuer,
//    2..5 = gather (one h slice each in flight), 6..9 = epilogue (TMEM lane
//    quarter warp % 4).  Weight stages, h slices and D buffers are rings
//    with full/empty mbarriers; every wait is bounded.
//  * MXFP8 weights (moe_down_tc_mx_kernel): the weight stages hold E4M3
//    boxes of 128 K-bytes x 128 rows (no swizzle) and each item's UE8M0
//    scales (128 rows x inter / 32 bytes, one bulk copy) sit in a ring of
//    two; eight more warps (10..17) decode each box into two bf16 K-chunks
//    of the 128-byte-swizzled layout in a ring of converted tiles (the
//    decode of the MXFP8 gate_up kernel) and free the E4M3 stage as soon as
//    it is decoded; the MMA reads A from the converted tiles.
#pragma once

#include "wd_down.cuh"
#include "wd_gate_up_tc.cuh"
#include "wd_tc.cuh"

namespace wdb {

constexpr int DTC_M = 128;                       // output rows per tile (MMA M)
constexpr int DTC_BK = 64;                       // K elements per chunk (128-byte rows)
constexpr int DTC_MAXKC = 32;                    // inter <= 2048
constexpr int DTC_SC = 4;                        // max K chunks per weight stage
constexpr int DTC_N = 16;                        // members per item (MMA N)
constexpr int DTC_ND = 4;                        // TMEM accumulator buffers
constexpr int DTC_GW = 4;                        // gather warps
constexpr int DTC_THREADS = (2 + DTC_GW + 4) * 32;
constexpr int DTC_A_CHUNK = DTC_M * DTC_BK * 2;  // 16 KB of weights
constexpr int DTC_B_CHUNK = DTC_N * DTC_BK * 2;  // 2 KB of h rows
constexpr uint32_t DTC_TMEM_COLS = DTC_ND * DTC_N < 32 ? 32 : DTC_ND * DTC_N;
constexpr int DTC_MX_CW = 8;                     // MXFP8 converter warps
constexpr int DTC_MX_THREADS = DTC_THREADS + DTC_MX_CW * 32;
constexpr int DTC_MX_BOX = DTC_M * 128;          // E4M3 box: 128 rows x 128 K (bytes)
constexpr int DTC_MX_NMAX = 16;                  // tokens per MXFP8 launch

// Fused all-reduce over the ranks of a tensor-parallel group (one process per
// GPU, peer memory opened through CUDA IPC).  Every rank's buffer holds
// [2 slots][world][max_tokens][H] packets of 8 bytes: the FP32 value in the
// low half and the epoch of the call that wrote it in the high half, stored
// and loaded as ONE 64-bit access (single-copy atomic), so a reader that sees
// the epoch sees the value that came with it (no fences, no separate flags).
// epochs[] counts this rank's calls: CTA c of a call reads epochs[c] and at
// the end writes the new count to epochs[c], epochs[c + grid], ..., so every
// entry advances by one per call whatever grid the kernel used (the
// single-launch FFN and the tensor-core down kernel partition the rows
// differently; a packet left by either never carries a current epoch).
// slot = epoch & 1 keeps a rank that is one call ahead off the slot still
// being read: a rank finishes call k + 1 only after hearing from every peer
// in call k + 1, and a peer's call k + 1 starts after its call k has ended.
//
// Two exchange shapes, the same result bits (every row is summed over the
// ranks' FP32 partials in rank order, then rounded to bf16 once):
//  * one-shot: every rank pushes its partial of every row to every rank and
//    sums all ranks' packets itself (one NVLink latency, B*H*8*(world-1)
//    bytes sent per rank);
//  * two-shot: row j is owned by rank (j/4) % world.  A rank pushes its partial
//    of a row to the owner only; the owner sums the packets in rank order
//    and pushes the bf16 result (as an FP32 packet) to the other ranks,
//    which take it from their own buffer at [owner][t][j] (two latencies,
//    about 2*B*H*8*(world-1)/world bytes per rank).
// Every push of a call precedes every wait of the same thread, owners sum
// before they gather, and all waits poll local memory only.
constexpr int TP_MAX_WORLD = 8;
struct TpArgs {
  int world;                        // <= 1: no fused all-reduce
  int rank;
  int max_tokens, max_ctas;
  int two_shot;                     // exchange shape (see above)
  unsigned long long* recv[TP_MAX_WORLD];  // packet buffers of every rank (peer pointers)
  uint32_t* epochs;                 // this rank's per-CTA call counters
};

// Packet accesses are scalar 64-bit volatile operations: PTX gives volatile
// global accesses the semantics of relaxed system-scope ones, so an aligned
// 64-bit access is single-copy atomic (a vector access would not be).  The
// explicit st/ld.relaxed.sys forms are equivalent but measured slower here
// (2 x B200, B = 16: 133.9 vs 104.6 us per tensor-parallel FFN call).
__device__ __forceinline__ void tp_put(unsigned long long* p, float v, uint32_t ep) {
  const unsigned long long w =
      ((unsigned long long)ep << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.volatile.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long tp_peek(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Four packets of consecutive rows in one 32-byte vector store (p 32-byte
// aligned): each 64-bit element is still one single-copy-atomic packet, and
// a warp's stores cover whole sectors instead of a quarter of each.
__device__ __forceinline__ void tp_put4(unsigned long long* p, const float (&v)[4], uint32_t ep) {
  const unsigned long long e = (unsigned long long)ep << 32;
  asm volatile("st.volatile.global.v4.b64 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "l"(e | __float_as_uint(v[0])), "l"(e | __float_as_uint(v[1])),
               "l"(e | __float_as_uint(v[2])), "l"(e | __float_as_uint(v[3]))
               : "memory");
}

// The value of the packet at p once it carries epoch ep; false if it did not
// arrive within WD_WAIT_LIMIT_NS.
__device__ __forceinline__ bool tp_take(const unsigned long long* p, uint32_t ep, float& v) {
  unsigned long long w = tp_peek(p);
  if ((uint32_t)(w >> 32) != ep) {
    const uint64_t t0 = globaltimer_ns();
    do {
      w = tp_peek(p);
      if ((uint32_t)(w >> 32) != ep && globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) return false;
    } while ((uint32_t)(w >> 32) != ep);
  }
  v = __uint_as_float((uint32_t)w);
  return true;
}

// One call's view of the exchange.
struct TpCall {
  const TpArgs& tp;
  uint32_t ep;  // this call's epoch
  int H;
  __device__ unsigned long long* at(int dst, int src, int t, int row) const {
    return tp.recv[dst] +
           (((size_t)((int)(ep & 1u) * tp.world + src) * tp.max_tokens + t) * H + row);
  }
  // The rank that sums `row` (every rank sums every row one-shot).  Two-shot:
  // four-row units dealt round robin, so every CTA sums about 1/world of its
  // rows on every rank (no rank's CTAs do all the summing).
  __device__ int owner(int row) const { return tp.two_shot ? (row >> 2) % tp.world : tp.rank; }
  __device__ bool sums(int row) const { return owner(row) == tp.rank; }
  // This rank's FP32 partial of (t, row) to the rank(s) that sum it.
  __device__ void push(int t, int row, float v) const {
    if (tp.two_shot) {
      tp_put(at(owner(row), tp.rank, t, row), v, ep);
    } else {
      for (int r = 0; r < tp.world; ++r) tp_put(at(r, tp.rank, t, row), v, ep);
    }
  }
  // This rank's partials of rows row..row + 3 of token t (row % 4 == 0, all
  // four below H; H % 4 == 0, so the packets are 32-byte aligned): one
  // vector store per destination rank.
  __device__ void push4(int t, int row, const float (&v)[4]) const {
    if (tp.two_shot) {
      tp_put4(at(owner(row), tp.rank, t, row), v, ep);
    } else {
      for (int r = 0; r < tp.world; ++r) tp_put4(at(r, tp.rank, t, row), v, ep);
    }
  }
  // The value of the packet at p, given a first reading w, once it carries
  // this call's epoch; false if it did not arrive within WD_WAIT_LIMIT_NS.
  __device__ bool settle(const unsigned long long* p, unsigned long long w, float& v) const {
    if ((uint32_t)(w >> 32) != ep) {
      const uint64_t t0 = globaltimer_ns();
      do {
        w = tp_peek(p);
        if ((uint32_t)(w >> 32) != ep && globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) return false;
      } while ((uint32_t)(w >> 32) != ep);
    }
    v = __uint_as_float((uint32_t)w);
    return true;
  }
  // The ranks' packets of (t, row) in this rank's buffer, read together.
  __device__ void peek_all(int t, int row, unsigned long long (&w)[TP_MAX_WORLD]) const {
#pragma unroll
    for (int r = 0; r < TP_MAX_WORLD; ++r)
      if (r < tp.world) w[r] = tp_peek(at(tp.rank, r, t, row));
  }
  // Sum of every rank's partial of (t, row) in rank order, from first
  // readings w (a row this rank sums; any late packet is polled); two-shot
  // also sends the bf16 result to the other ranks.
  __device__ bool reduce(int t, int row, const unsigned long long (&w)[TP_MAX_WORLD],
                         __nv_bfloat16& y) const {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < TP_MAX_WORLD; ++r) {
      if (r < tp.world) {
        float v;
        if (!settle(at(tp.rank, r, t, row), w[r], v)) return false;
        s += v;
      }
    }
    y = __float2bfloat16_rn(s);
    if (tp.two_shot) {
      const float yf = __bfloat162float(y);
      for (int r = 0; r < tp.world; ++r)
        if (r != tp.rank) tp_put(at(r, tp.rank, t, row), yf, ep);
    }
    return true;
  }
};

// This rank's output rows of the call after its pushes: entry i (i =
// threadIdx.x, + blockDim.x, ... < n) is (t, row) = entry(i), skipped where
// entry() returns false.  First the rows this rank sums (all one-shot), then
// (two-shot) the other rows from their owners; the packets of four (sums)
// or eight (owners' results) entries per thread are in flight together.  A
// packet that does not arrive within the bound gives a zero and raises
// WD_STATUS_WAIT_TIMEOUT; returns false then.
template <class Entry>
__device__ inline bool tp_collect(const TpCall& xc, int n, Entry entry, __nv_bfloat16* y,
                                  uint32_t* status) {
  bool ok = true;
  const __nv_bfloat16 zero = __float2bfloat16_rn(0.f);
  constexpr int RB = 4;  // entries per thread whose packets are in flight together
  for (int i0 = threadIdx.x; i0 < n; i0 += RB * (int)blockDim.x) {
    int tt[RB], rr[RB];
    bool take[RB];
    unsigned long long w[RB][TP_MAX_WORLD];
#pragma unroll
    for (int j = 0; j < RB; ++j) {
      const int i = i0 + j * (int)blockDim.x;
      take[j] = i < n && entry(i, tt[j], rr[j]) && xc.sums(rr[j]);
      if (take[j]) xc.peek_all(tt[j], rr[j], w[j]);
    }
#pragma unroll
    for (int j = 0; j < RB; ++j) {
      if (!take[j]) continue;
      __nv_bfloat16 yv = zero;
      if (ok && !xc.reduce(tt[j], rr[j], w[j], yv)) {
        ok = false;
        yv = zero;
        raise_status(status, WD_STATUS_WAIT_TIMEOUT);
      }
      y[(size_t)tt[j] * xc.H + rr[j]] = yv;
    }
  }
  if (!xc.tp.two_shot) return ok;
  constexpr int GB = 8;
  for (int i0 = threadIdx.x; i0 < n; i0 += GB * (int)blockDim.x) {
    int tt[GB], rr[GB];
    bool take[GB];
    unsigned long long w[GB];
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      const int i = i0 + j * (int)blockDim.x;
      take[j] = i < n && entry(i, tt[j], rr[j]) && !xc.sums(rr[j]);
      if (take[j]) w[j] = tp_peek(xc.at(xc.tp.rank, xc.owner(rr[j]), tt[j], rr[j]));
    }
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      if (!take[j]) continue;
      __nv_bfloat16 yv = zero;
      float v;
      if (ok) {
        if (xc.settle(xc.at(xc.tp.rank, xc.owner(rr[j]), tt[j], rr[j]), w[j], v)) {
          yv = __float2bfloat16_rn(v);
        } else {
          ok = false;
          raise_status(status, WD_STATUS_WAIT_TIMEOUT);
        }
      }
      y[(size_t)tt[j] * xc.H + rr[j]] = yv;
    }
  }
  return ok;
}

struct DownTcArgs {
  const __nv_bfloat16* h;  // [B*K, I]
  const int32_t* ids;      // [B, K]
  const float* scale;      // [B, K]
  void* out;               // [B, H] bf16 or fp32
  int out_fp32;
  uint32_t* status;
  int B, E, K, H, I;
  int stages;              // weight ring depth
  int sc;                  // K chunks per weight stage (<= DTC_SC)
  int nbuf;                // h slices (the K range of one weight stage of one
                           // item), >= DTC_GW (a gather warp is at most one
                           // ring turn ahead, so mbarrier parities cannot alias)
  int cl;                  // CTAs per cluster (1 to 8)
  TpArgs tp;               // fused all-reduce (tp.world > 1): out = bf16 sum over ranks
  const uint8_t* wscale;   // MXFP8: UE8M0 scales [E, H, I / 32] (nullptr for bf16)
  int conv;                // MXFP8: converted-box ring depth
};

__host__ __device__ inline int down_tc_kc(int I) { return (I + DTC_BK - 1) / DTC_BK; }

__host__ inline int down_tc_smem_bytes(int stages, int sc, int nbuf, int I, int B, int n, int E) {
  const int kc = down_tc_kc(I);
  (void)kc;
  return 1024 + stages * sc * DTC_A_CHUNK + nbuf * sc * DTC_B_CHUNK + B * DTC_M * 4 +
         ((n * 4 + 127) / 128) * 128 + (2 * stages + 2 * nbuf + 2 * DTC_ND + 1) * 8 + 16 +
         CTRL_INTS * 4 + route_smem_bytes(n, E, true);
}

// MXFP8: weight stages of sc / 2 E4M3 boxes, two scale slots of 4 * I bytes,
// `conv` converted boxes; the rest as for bf16.
__host__ inline int down_tc_mx_smem_bytes(int stages, int sc, int nbuf, int conv, int I, int B,
                                          int n, int E) {
  return 1024 + stages * (sc / 2) * DTC_MX_BOX + nbuf * sc * DTC_B_CHUNK + conv * TC_MX_CONV +
         2 * 4 * I + B * DTC_M * 4 + ((n * 4 + 127) / 128) * 128 +
         (2 * stages + 2 * nbuf + 2 * DTC_ND + 1 + 2 * conv + 4) * 8 + 16 + CTRL_INTS * 4 +
         route_smem_bytes(n, E, true);
}

// Body of both kernels.  kTP: the fused all-reduce variant (tp.world > 1);
// the plain kernel carries none of its code.  kMx: MXFP8 weights.  kRoute:
// routing code compiled for this launch's slot count (RouteMode).
// kFused: phase 2 of moe_ffn_tc_kernel (FusedCtx: shared-memory region,
// routing, top-k weights and TMEM given; h is written by the other CTAs of
// the same launch, so the gather warps wait for the grid barrier and read h
// through L2).  The weight stream starts before that wait.
template <bool kTP, bool kMx, int kRoute, bool kFused = false>
__device__ __forceinline__ void down_tc_body(const CUtensorMap& tm_w, const DownTcArgs a,
                                             const FusedCtx* fx = nullptr) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = kFused ? fx->base : smem_raw + pad;
  const int S = a.stages, NB = a.nbuf, CL = a.cl;
  const int I = a.I;
  const int kc = down_tc_kc(I);
  const int n = a.B * a.K;
  const int SC = a.sc;              // K chunks per weight stage
  const int nst = (kc + SC - 1) / SC;  // weight stages per item
  const int SB = kMx ? (SC / 2) * DTC_MX_BOX : SC * DTC_A_CHUNK;  // bytes of one weight stage
  const int BB = SC * DTC_B_CHUNK;  // bytes of one h slice (one weight stage's K range)
  const int CS = kMx ? a.conv : 0;
  const int SCB = kMx ? 4 * I : 0;  // MXFP8: bytes of one item's scales (128 rows x I / 32)
  uint8_t* wring = base;
  uint8_t* bring = wring + (size_t)S * SB;
  uint8_t* conv = bring + (size_t)NB * BB;  // MXFP8: [CS] converted boxes
  uint8_t* sring = conv + (size_t)CS * TC_MX_CONV;  // MXFP8: [2] item scales
  float* Y = reinterpret_cast<float*>(sring + 2 * SCB);  // [B][128]
  float* s_scale = kFused ? const_cast<float*>(fx->s_scale) : Y + a.B * DTC_M;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(Y + a.B * DTC_M + ((n * 4 + 127) / 128) * 32);
  uint64_t* wempty = wfull + S;
  uint64_t* bfull = wempty + S;
  uint64_t* bempty = bfull + NB;
  uint64_t* dfull = bempty + NB;
  uint64_t* dempty = dfull + DTC_ND;
  uint64_t* done = dempty + DTC_ND;
  uint64_t* cfull = done + 1;      // MXFP8: [CS] converted box written
  uint64_t* cempty = cfull + CS;   // MXFP8: [CS] converted box read by the MMAs
  uint64_t* sfull = cempty + CS;   // MXFP8: [2] item scales landed
  uint64_t* sempty = sfull + (kMx ? 2 : 0);  // MXFP8: [2] item scales decoded
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty + (kMx ? 2 : 0));
  volatile int* ctrl = reinterpret_cast<volatile int*>(tmem_slot + 4);
  int* route_base = const_cast<int*>(ctrl) + CTRL_INTS;
  const RouteSmem r = kFused ? *fx->r : route_carve(route_base, n, a.E, true);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = CL > 1 ? (int)cluster_ctarank() : 0;
  const int j0 = ((int)blockIdx.x / CL) * DTC_M;
  const uint32_t tp_ep = kTP && a.tp.world > 1 ? a.tp.epochs[blockIdx.x] + 1u : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kMx ? DTC_MX_CW : 1);  // MXFP8: freed by the converters
    }
    if constexpr (kMx) {
      for (int c = 0; c < CS; ++c) {
        mbar_init(&cfull[c], DTC_MX_CW);
        mbar_init(&cempty[c], 1);
      }
      for (int c = 0; c < 2; ++c) {
        mbar_init(&sfull[c], 1);
        mbar_init(&sempty[c], DTC_MX_CW);
      }
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&bfull[b], 1);
      mbar_init(&bempty[b], 1);
    }
    for (int d = 0; d < DTC_ND; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 4);
    }
    mbar_init(done, 1);
    ctrl[0] = 0;
    fence_mbar_init();
  }
  if (threadIdx.x == 32) prefetch_tensormap(&tm_w);
  if (!kFused && warp == 1) {
    tmem_alloc(tmem_slot, DTC_TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  for (int i = threadIdx.x; i < a.B * DTC_M; i += blockDim.x) Y[i] = 0.f;
  if constexpr (kFused) {
    __syncthreads();
  } else {
    // h, topk_scale (and possibly topk_ids) come from the preceding kernel.
    pdl_wait_primary();
    route_build<true, NoInit, kRoute>(r, a.ids, n, a.E, a.K, true, DTC_N, a.status, NoInit(),
                                      a.scale, s_scale);  // ends with __syncthreads
  }
  tc_fence_after();
  const uint32_t tmem = kFused ? fx->tmem : *tmem_slot;
  const int nsg = *r.nsg;

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
  // Items of this CTA: the valid groups rank, rank + CL, ... (the same
  // sequence in every role).
  auto next_item = [&](int g) {
    for (g += CL; g < nsg && r.sg_exp[g] < 0; g += CL) {
    }
    return g;
  };
  int g_first = rank;
  while (g_first < nsg && r.sg_exp[g_first] < 0) g_first += CL;

  if (warp == 0) {
    // ---------------- weight producer ----------------
    const uint64_t pol = l2_policy_evict_first();
    uint32_t it = 0;
    uint32_t ni = 0, nsi = 0;  // MXFP8: items started, scale copies issued
    bool ok = true;
    if (!kMx && nst == 1) {
      // one stage per item (inter <= 256)
      for (int g = g_first; g < nsg; g = next_item(g)) {
        const int slot = (int)(it % (uint32_t)S);
        if (lane == 0) {
          if (!wait(&wempty[slot], ((it / (uint32_t)S) & 1u) ^ 1u)) {
            ok = false;
          } else {
            uint8_t* st = wring + (size_t)slot * SB;
            mbar_arrive_expect_tx(&wfull[slot], (uint32_t)(kc * DTC_A_CHUNK));
            for (int c = 0; c < kc; ++c)
              tma_load_3d(st + c * DTC_A_CHUNK, &tm_w, c * DTC_BK, j0, r.sg_exp[g], &wfull[slot],
                          pol);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++it;
      }
    } else
    for (int g = g_first; ok && g < nsg; g = next_item(g), ++ni) {
      if constexpr (kMx) {
        // The item's scales: rows [j0, j0 + 128) x I / 32 bytes, contiguous.
        if (lane == 0) {
          const int sb = (int)(ni & 1u);
          if (!wait(&sempty[sb], ((ni >> 1) & 1u) ^ 1u)) {
            ok = false;
          } else {
            mbar_arrive_expect_tx(&sfull[sb], (uint32_t)SCB);
            bulk_g2s(sring + (size_t)sb * SCB,
                     a.wscale + ((size_t)r.sg_exp[g] * a.H + j0) * (size_t)(I / 32), (uint32_t)SCB,
                     &sfull[sb], pol);
            nsi = ni + 1;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      for (int sj = 0; sj < nst; ++sj) {
        const int slot = (int)(it % (uint32_t)S);
        const int c0 = sj * SC, nc = min(SC, kc - c0);
        if (lane == 0) {
          if (!wait(&wempty[slot], ((it / (uint32_t)S) & 1u) ^ 1u)) {
            ok = false;
          } else if constexpr (kMx) {
            // nc / 2 E4M3 boxes of 128 K-bytes (inter % 128 == 0 on this path)
            uint8_t* st = wring + (size_t)slot * SB;
            mbar_arrive_expect_tx(&wfull[slot], (uint32_t)((nc / 2) * DTC_MX_BOX));
            for (int b = 0; b < nc / 2; ++b)
              tma_load_3d(st + b * DTC_MX_BOX, &tm_w, (c0 + 2 * b) * DTC_BK, j0, r.sg_exp[g],
                          &wfull[slot], pol);
          } else {
            uint8_t* st = wring + (size_t)slot * SB;
            mbar_arrive_expect_tx(&wfull[slot], (uint32_t)(nc * DTC_A_CHUNK));
            for (int c = 0; c < nc; ++c)
              tma_load_3d(st + c * DTC_A_CHUNK, &tm_w, (c0 + c) * DTC_BK, j0, r.sg_exp[g],
                          &wfull[slot], pol);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++it;
      }
    }
    if (!ok && lane == 0) {
      const uint32_t lo = it > (uint32_t)S ? it - (uint32_t)S : 0u;
      for (uint32_t i = lo; i < it; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&wfull[i % (uint32_t)S], (i / (uint32_t)S) & 1u) &&
               globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
        }
      }
      if constexpr (kMx) {
        const uint32_t slo = nsi > 2u ? nsi - 2u : 0u;
        for (uint32_t i = slo; i < nsi; ++i) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&sfull[i & 1u], (i >> 1) & 1u) &&
                 globaltimer_ns() - t0 < WD_WAIT_LIMIT_NS) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, its = 0, ci = 0;  // items, weight stages, converted boxes
      bool issued = false, ok = true;
      const uint32_t idesc = tc_idesc_bf16(DTC_M, DTC_N);
      if (!kMx && nst == 1) {
        // one stage per item (inter <= 256)
        for (int g = g_first; g < nsg; g = next_item(g)) {
          const int slot = (int)(it % (uint32_t)S);
          const int bb = (int)(it % (uint32_t)NB);
          const int d = (int)(it % (uint32_t)DTC_ND);
          if (!wait(&wfull[slot], (it / (uint32_t)S) & 1u) ||
              !wait(&bfull[bb], (it / (uint32_t)NB) & 1u) ||
              !wait(&dempty[d], ((it / (uint32_t)DTC_ND) & 1u) ^ 1u))
            break;
          tc_fence_after();
          const uint8_t* W = wring + (size_t)slot * SB;
          const uint8_t* Bt = bring + (size_t)bb * BB;
          const uint32_t dt = tmem + (uint32_t)(d * DTC_N);
          for (int c = 0; c < kc; ++c) {
            const uint64_t ad = tc_desc_sw128(smem_u32(W + c * DTC_A_CHUNK));
            const uint64_t bd = tc_desc_sw128(smem_u32(Bt + c * DTC_B_CHUNK));
#pragma unroll
            for (int kk = 0; kk < DTC_BK / 16; ++kk)
              tc_mma_bf16(dt, ad + 2u * kk, bd + 2u * kk, idesc, (c | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&wempty[slot]);
          tc_commit(&bempty[bb]);
          tc_commit(&dfull[d]);
          issued = true;
          ++it;
        }
      } else
      for (int g = g_first; ok && g < nsg; g = next_item(g)) {
        const int d = (int)(it % (uint32_t)DTC_ND);
        if (!wait(&dempty[d], ((it / (uint32_t)DTC_ND) & 1u) ^ 1u)) break;
        const uint32_t dt = tmem + (uint32_t)(d * DTC_N);
        for (int sj = 0; sj < nst; ++sj, ++its) {
          const int slot = (int)(its % (uint32_t)S);
          const int hb = (int)(its % (uint32_t)NB);
          const int c0 = sj * SC, nc = min(SC, kc - c0);
          if constexpr (kMx) {
            // A from the converted boxes of this stage (two K-chunks each),
            // B from the stage's h slice; the converters free the E4M3 stage.
            if (!wait(&bfull[hb], (its / (uint32_t)NB) & 1u)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint8_t* Bt = bring + (size_t)hb * BB;
            for (int b = 0; b < nc / 2; ++b, ++ci) {
              const int cs = (int)(ci % (uint32_t)CS);
              if (!wait(&cfull[cs], (ci / (uint32_t)CS) & 1u)) { ok = false; break; }
              tc_fence_after();
              for (int hh = 0; hh < 2; ++hh) {
                const int cc = 2 * b + hh;
                const uint64_t ad =
                    tc_desc_sw128(smem_u32(conv + (size_t)cs * TC_MX_CONV + hh * DTC_A_CHUNK));
                const uint64_t bd = tc_desc_sw128(smem_u32(Bt + cc * DTC_B_CHUNK));
#pragma unroll
                for (int kk = 0; kk < DTC_BK / 16; ++kk)
                  tc_mma_bf16(dt, ad + 2u * kk, bd + 2u * kk, idesc,
                              ((c0 + cc) | kk) != 0 ? 1u : 0u);
              }
              tc_commit(&cempty[cs]);
              issued = true;
            }
            if (!ok) break;
            tc_commit(&bempty[hb]);
          } else {
            if (!wait(&wfull[slot], (its / (uint32_t)S) & 1u) ||
                !wait(&bfull[hb], (its / (uint32_t)NB) & 1u)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint8_t* W = wring + (size_t)slot * SB;
            const uint8_t* Bt = bring + (size_t)hb * BB;
            for (int cc = 0; cc < nc; ++cc) {
              const uint64_t ad = tc_desc_sw128(smem_u32(W + cc * DTC_A_CHUNK));
              const uint64_t bd = tc_desc_sw128(smem_u32(Bt + cc * DTC_B_CHUNK));
#pragma unroll
              for (int kk = 0; kk < DTC_BK / 16; ++kk)
                tc_mma_bf16(dt, ad + 2u * kk, bd + 2u * kk, idesc,
                            ((c0 + cc) | kk) != 0 ? 1u : 0u);
            }
            tc_commit(&wempty[slot]);
            tc_commit(&bempty[hb]);
            issued = true;
          }
        }
        if (!ok) break;
        tc_commit(&dfull[d]);
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
  } else if (warp < 2 + DTC_GW) {
    // -------- gather: h slice of stage its (K range of one weight stage of
    // one item), warp its % DTC_GW --------
    const int gw = warp - 2;
    const int vecs = I / 8;  // 16-byte pieces per h row
    uint32_t its = 0;
    bool got = true;
    if constexpr (kFused) {
      // h of the whole launch: every CTA has added its arrivals after its
      // gate_up phase (release); wait for all of them (acquire, bounded).
      if (gw == 0 && lane == 0) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu_u64(fx->sync) < fx->target) {
          if (globaltimer_ns() - t0 > WD_WAIT_LIMIT_NS) {
            raise_status(a.status, WD_STATUS_WAIT_TIMEOUT);
            ctrl[0] = 1;
            break;
          }
          __nanosleep(32);
        }
      }
      named_barrier_sync(3, 32 * DTC_GW);
    }
    auto ldh = [&](const __nv_bfloat16* p) { return kFused ? ldcg16(p) : ldg16(p); };
    if (!kMx && nst == 1) {
      // one slice per item (inter <= 256): the item loop alone
      for (int g = g_first; g < nsg; g = next_item(g), ++its) {
        if ((int)(its % DTC_GW) != gw) continue;
        const int hb = (int)(its % (uint32_t)NB);
        got = __all_sync(0xffffffffu, wait(&bempty[hb], ((its / (uint32_t)NB) & 1u) ^ 1u));
        if (!got) break;
        const int beg = r.sg_beg[g], cnt = r.sg_cnt[g];
        uint8_t* Bt = bring + (size_t)hb * BB;
        for (int pc = lane; pc < cnt * kc * 8; pc += 32) {
          const int p = pc / (kc * 8), rem = pc - p * (kc * 8);
          const int c = rem >> 3, j = rem & 7;
          const int kv = c * 8 + j;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (kv < vecs) v = ldh(a.h + (size_t)r.members[beg + p] * I + kv * 8);
          *reinterpret_cast<uint4*>(Bt + c * DTC_B_CHUNK + (p >> 3) * 1024 + (p & 7) * 128 +
                                    ((j ^ (p & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[hb]);
      }
    } else
    for (int g = g_first; got && g < nsg; g = next_item(g)) {
      const int beg = r.sg_beg[g], cnt = r.sg_cnt[g];
      for (int sj = 0; sj < nst; ++sj, ++its) {
        if ((int)(its % DTC_GW) != gw) continue;
        const int hb = (int)(its % (uint32_t)NB);
        got = __all_sync(0xffffffffu, wait(&bempty[hb], ((its / (uint32_t)NB) & 1u) ^ 1u));
        if (!got) break;
        const int c0 = sj * SC, nc = min(SC, kc - c0);
        uint8_t* Bt = bring + (size_t)hb * BB;
        for (int pc = lane; pc < cnt * nc * 8; pc += 32) {
          const int p = pc / (nc * 8), rem = pc - p * (nc * 8);
          const int c = rem >> 3, j = rem & 7;
          const int kv = (c0 + c) * 8 + j;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (kv < vecs) v = ldh(a.h + (size_t)r.members[beg + p] * I + kv * 8);
          *reinterpret_cast<uint4*>(Bt + c * DTC_B_CHUNK + (p >> 3) * 1024 + (p & 7) * 128 +
                                    ((j ^ (p & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[hb]);
      }
    }
  } else if (warp < 2 + DTC_GW + 4) {
    // ---------------- epilogue: row j = 32 * (warp % 4) + lane ------------
    const int q = warp & 3;
    const int j = 32 * q + lane;
    uint32_t it = 0;
    for (int g = g_first; g < nsg; g = next_item(g), ++it) {
      const int d = (int)(it % (uint32_t)DTC_ND);
      // Warp-uniform decision: tcgen05.ld below is warp-collective.
      const bool got = __all_sync(0xffffffffu, wait(&dfull[d], (it / (uint32_t)DTC_ND) & 1u));
      if (!got) break;
      tc_fence_after();
      uint32_t v[16];
      tmem_ld_x16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(d * DTC_N), v);
      tmem_wait_ld();
      const int beg = r.sg_beg[g], cnt = r.sg_cnt[g];
#pragma unroll
      for (int c = 0; c < DTC_N; ++c) {
        if (c < cnt) {
          const int p = beg + c;
          float* y = Y + r.mtok[p] * DTC_M + j;
          *y = fmaf(s_scale[r.members[p]], __uint_as_float(v[c]), *y);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
    }
  } else {
    // ---------------- MXFP8 converters: warps 10..17 (mx_convert_box) ----
    // Scale byte of (row, K block kb): sring[row * (I / 32) + kb].
    if constexpr (kMx) {
    static_assert(DTC_MX_CW == TC_MX_CW && DTC_M == TC_M, "shared box converter");
    const int cw = warp - (2 + DTC_GW + 4);
    const int nb = I / 32;
    uint32_t its = 0, ci = 0, ni = 0;
    bool ok = true;
    for (int g = g_first; ok && g < nsg; g = next_item(g), ++ni) {
      const int sb = (int)(ni & 1u);
      if (!wait(&sfull[sb], (ni >> 1) & 1u)) break;
      const uint8_t* sc = sring + (size_t)sb * SCB;
      for (int sj = 0; sj < nst; ++sj, ++its) {
        const int slot = (int)(its % (uint32_t)S);
        if (!wait(&wfull[slot], (its / (uint32_t)S) & 1u)) { ok = false; break; }
        const int c0 = sj * SC, nc = min(SC, kc - c0);
        const uint8_t* w8 = wring + (size_t)slot * SB;
        for (int b = 0; b < nc / 2; ++b, ++ci) {
          const int cs = (int)(ci % (uint32_t)CS);
          if (!wait(&cempty[cs], ((ci / (uint32_t)CS) & 1u) ^ 1u)) { ok = false; break; }
          const int kb0 = 2 * (c0 + 2 * b);  // first 32-element block of the box
          mx_convert_box(w8 + b * DTC_MX_BOX, conv + (size_t)cs * TC_MX_CONV, sc + kb0, nb, cw,
                         lane);
          fence_proxy_async_smem();  // generic writes -> tensor-core reads
          __syncwarp();
          if (lane == 0) mbar_arrive(&cfull[cs]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[slot]);  // E4M3 stage decoded
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[sb]);  // item scales no longer read
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Y is final: release it to the cluster, free TMEM meanwhile, then sum the
  // CL partial tiles in rank order; CTA `rank` writes rows [lo, hi) of the
  // tile (the 32 four-row units split as evenly as CL allows; CL need not
  // divide 128), 4 rows per thread.
  if (CL > 1) cluster_arrive();
  if (!kFused && warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, DTC_TMEM_COLS);
  }
  if (CL > 1) cluster_wait();
  const int lo = (rank * (DTC_M / 4) / CL) * 4;
  const int hi = ((rank + 1) * (DTC_M / 4) / CL) * 4;
  const int q4 = (hi - lo) / 4;
  const bool tp = kTP && a.tp.world > 1;
  const TpCall xc{a.tp, tp_ep, a.H};  // this call's exchange (tp only)
  for (int i = threadIdx.x; i < a.B * q4; i += blockDim.x) {
    const int t = i / q4, jj = lo + 4 * (i - t * q4);
    const float* src = &Y[t * DTC_M + jj];
    float4 acc;
    if (CL > 1) {
      float4 part[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < CL) part[k] = dsmem_ld_f32x4(dsmem_addr(src, (uint32_t)k));
      acc = part[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) {
        if (k < CL) {
          acc.x += part[k].x; acc.y += part[k].y; acc.z += part[k].z; acc.w += part[k].w;
        }
      }
    } else {
      acc = *reinterpret_cast<const float4*>(src);
    }
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if constexpr (kTP) if (tp) {
      // This rank's partials of the rows go out first (no wait in between).
      if (j0 + jj + 3 < a.H && (a.H & 3) == 0) {
        xc.push4(t, j0 + jj, v);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + jj + u < a.H) xc.push(t, j0 + jj + u, v[u]);
      }
      continue;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int row = j0 + jj + u;
      if (row < a.H) {
        if (a.out_fp32)
          reinterpret_cast<float*>(a.out)[(size_t)t * a.H + row] = v[u];
        else
          reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.H + row] =
              __float2bfloat16_rn(v[u]);
      }
    }
  }
  if constexpr (kTP) if (tp) {
    const int nr = hi - lo;
    tp_collect(xc, a.B * nr, [&](int i, int& t, int& row) {
      t = i / nr;
      row = j0 + lo + (i - t * nr);
      return row < a.H;
    }, reinterpret_cast<__nv_bfloat16*>(a.out), a.status);
  }
  if (tp && threadIdx.x == 0)
    for (int c2 = (int)blockIdx.x; c2 < a.tp.max_ctas; c2 += (int)gridDim.x) a.tp.epochs[c2] = tp_ep;
  if (CL > 1) cluster_sync();  // no CTA leaves while a peer may read its tile
}

template <bool kTP, int kRoute>
__global__ void __launch_bounds__(DTC_THREADS, 1)
    moe_down_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const DownTcArgs a) {
  down_tc_body<kTP, false, kRoute>(tm_w, a);
}

// MXFP8 weights: tm_w over the E4M3 bytes [E, H, I], a.wscale the UE8M0
// scales [E, H, I / 32].  Single GPU (no fused all-reduce).
template <int kRoute>
__global__ void __launch_bounds__(DTC_MX_THREADS, 1)
    moe_down_tc_mx_kernel(const __grid_constant__ CUtensorMap tm_w, const DownTcArgs a) {
  down_tc_body<false, true, kRoute>(tm_w, a);
}

}  // namespace wdb
