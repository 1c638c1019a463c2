// C ABI of warp_decode_b200: argument validation, launch geometry and
// dispatch for the fused MoE decode kernels.  Single translation unit so the
// library-owned status word needs no relocatable device code.
//
// Host-side behaviour mirrors the reference binding (csrc/binding.cpp:35-121):
// shapes are checked before anything is launched, the output is written on
// the caller's stream, nothing synchronises.  Differences: errors are return
// codes (the torch layer turns them into RuntimeError), expert ids are
// range-checked on the device, and B = 0 is a valid no-op.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include <array>
#include <atomic>
#include <cmath>
#include <vector>

#include "wd_down.cuh"
#include "wd_gate_up.cuh"
#include "wd_gate_up_tc.cuh"
#include "wd_down_tc.cuh"
#include "wd_ffn.cuh"
#include "wd_ffn_tc.cuh"
#include "wd_router.cuh"
#include "wd_copy.cuh"

// Scratch of wd_moe_ffn_3d_batched_noalloc: [0, 8) the grid-barrier counter
// (zero at module load; each single-launch call adds GRID_BAR_UNITS in total,
// so it never needs resetting), [256, 256 + 128 KiB) h of the call
// (B*topk*inter bf16, e.g. 64 routed slots x 1024 inter).  One copy per device; calls that overlap
// in time race on it.
constexpr size_t kNoallocHeader = 256;
constexpr size_t kNoallocHBytes = (size_t)64 * 1024 * 2;
static __device__ __align__(256) unsigned char g_wd_noalloc_scratch[kNoallocHeader + kNoallocHBytes];

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

// Kernels enqueued by this library in this process (wd_launch_count).
std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sm_count = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;      // shared memory of one SM
  int smem_reserved = 0;    // shared memory the runtime reserves per CTA
  unsigned long long* ffn_sync = nullptr;  // library-owned grid-barrier counter (g_wd_ffn_sync)
  unsigned char* noalloc_scratch = nullptr;  // g_wd_noalloc_scratch, set on first use
  std::atomic<bool> ffn_tc_off{false};  // moe_ffn_tc_kernel's launch was refused once
  bool ready = false;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

// Per-device setup: SM count, opt-in shared memory and kernel attributes.
// Runs once per device, on the first call made with that device current.
int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(WD_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return fail(WD_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    err = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (err == cudaSuccess)
      err = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (err == cudaSuccess)
      err = cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (err == cudaSuccess)
      err = cudaDeviceGetAttribute(&d.smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    const void* kernels[] = {
        reinterpret_cast<const void*>(&wdb::moe_gate_up_kernel<wdb::W_BF16, wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_kernel<wdb::W_BF16, wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_kernel<wdb::W_E4M3, wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_kernel<wdb::W_E4M3, wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_down_kernel<wdb::W_BF16, wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_down_kernel<wdb::W_BF16, wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_down_kernel<wdb::W_E4M3, wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_down_kernel<wdb::W_E4M3, wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_tc_kernel<wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_tc_kernel<wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_tc_mx_kernel<wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_gate_up_tc_mx_kernel<wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_down_tc_kernel<false, wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_down_tc_kernel<false, wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_down_tc_kernel<true, wdb::ROUTE_ANY>),
        reinterpret_cast<const void*>(&wdb::moe_down_tc_mx_kernel<wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_down_tc_mx_kernel<wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_ffn_kernel<false>),
        reinterpret_cast<const void*>(&wdb::moe_ffn_kernel<true>),
        reinterpret_cast<const void*>(&wdb::moe_ffn_tc_kernel<wdb::ROUTE_SMALL>),
        reinterpret_cast<const void*>(&wdb::moe_ffn_tc_kernel<wdb::ROUTE_LARGE>),
        reinterpret_cast<const void*>(&wdb::moe_ffn_tc_kernel<wdb::ROUTE_ANY, true>),
    };
    for (const void* k : kernels) {
      if (err != cudaSuccess) break;
      // Dynamic + static shared memory must fit the opt-in limit; the kernels
      // use well under 1 KB of static shared memory.
      err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 d.smem_optin - 1024);
      // Full shared-memory carve-out so a gate_up CTA and an early-started
      // down CTA fit on one SM together.
      if (err == cudaSuccess)
        err = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                   (int)cudaSharedmemCarveoutMaxShared);
    }
    if (err == cudaSuccess)
      err = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.ffn_sync), wdb::g_wd_ffn_sync);
    if (err != cudaSuccess)
      return fail(WD_ERR_CUDA, std::string("device setup: ") + cudaGetErrorString(err));
    d.ready = true;
  }
  *out = &d;
  return WD_OK;
}

// Programmatic dependent launch of down behind gate_up: opt-in
// (WARP_DECODE_PDL=1).  Measured on B200 with CUDA-graph replay: with gate_up
// triggering at its entry the pair was slower (B=2: 43.1 vs 35.0 us, B=4:
// 53.5 vs 47.1, B=8: 64.7 vs 61.9) -- the down CTAs cannot share an SM with a
// gate_up CTA (shared memory), and the early-launched grid delays its
// clusters; with the trigger after each gate_up CTA's last h store (now) it
// is level or a little ahead (B=6: 53.2 vs 53.4 us, B=8: 61.4 vs 61.9), too
// little to make it the default.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WARP_DECODE_PDL");
    return v && v[0] == '1';
  }();
  return on;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int B, int E, int topk, int hidden, int inter) {
  if (B < 0) return fail(WD_ERR_SHAPE, "B must be >= 0");
  if (E < 1) return fail(WD_ERR_SHAPE, "E (number of experts) must be >= 1");
  if (topk < 1) return fail(WD_ERR_SHAPE, "topk must be >= 1");
  if (topk > wdb::MAX_SLOTS) return fail(WD_ERR_UNSUPPORTED, "topk must be <= 512");
  if (hidden < 1 || inter < 1) return fail(WD_ERR_SHAPE, "hidden and inter must be >= 1");
  return WD_OK;
}

// ---- gate_up path selection -------------------------------------------------
// 0 = automatic (tensor cores from WD_TC_MIN_TOKENS tokens per launch),
// 1 = SIMT kernel only, 2 = tensor-core kernel wherever it applies.
#ifndef WD_TC_MIN_TOKENS
#define WD_TC_MIN_TOKENS 16
#endif
#ifndef WD_DTC_MIN_TOKENS
#define WD_DTC_MIN_TOKENS 2
#endif
// MXFP8 weights: tensor cores (on-chip E4M3 decode) from this many tokens.
// Measured gate_up (H 2048, I 768, E 128, top-8, cold, B200), tensor cores vs
// SIMT: B = 2 34.9 vs 32.7 us, B = 4 47.2 vs 57.2, B = 8 74.8 vs 96.3,
// B = 16 106.5 vs 174.8.
#ifndef WD_TC_MX_MIN_TOKENS
#define WD_TC_MX_MIN_TOKENS 4
#endif
#ifndef WD_TC_KCH
#define WD_TC_KCH 4
#endif
#ifndef WD_TC_L2PROMO
#define WD_TC_L2PROMO CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif
std::atomic<int> g_gate_up_path{-1};
std::atomic<int> g_down_path{-1};

// Current choice of one kernel's path; the first call reads the environment.
int kernel_path(std::atomic<int>& slot, const char* env) {
  int p = slot.load(std::memory_order_relaxed);
  if (p < 0) {
    const char* v = std::getenv(env);
    p = 0;
    if (v && std::strcmp(v, "simt") == 0) p = 1;
    if (v && std::strcmp(v, "tc") == 0) p = 2;
    int expected = -1;
    slot.compare_exchange_strong(expected, p);
    p = slot.load(std::memory_order_relaxed);
  }
  return p;
}

int gate_up_path() { return kernel_path(g_gate_up_path, "WARP_DECODE_GATE_UP"); }
int down_path() { return kernel_path(g_down_path, "WARP_DECODE_DOWN"); }

// FFN entry point: 0 = automatic (SIMT single launch up to
// WD_FFN_AUTO_MAX_SLOTS routed slots, the tensor-core single launch above
// where it applies), 1 = always the two kernels, 2 = SIMT single launch
// wherever it applies (up to 64 routed slots), 3 = tensor-core single launch
// wherever it applies.
// WARP_DECODE_FFN=split|fused|tc sets the initial choice.
std::atomic<int> g_ffn_path{-1};
int ffn_path() {
  int p = g_ffn_path.load(std::memory_order_relaxed);
  if (p < 0) {
    const char* v = std::getenv("WARP_DECODE_FFN");
    p = 0;
    if (v && std::strcmp(v, "split") == 0) p = 1;
    if (v && std::strcmp(v, "fused") == 0) p = 2;
    if (v && std::strcmp(v, "tc") == 0) p = 3;
    int expected = -1;
    g_ffn_path.compare_exchange_strong(expected, p);
    p = g_ffn_path.load(std::memory_order_relaxed);
  }
  return p;
}

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

#ifndef WD_TC_MAX_CLUSTER
#define WD_TC_MAX_CLUSTER 8
#endif

// How many clusters of `cl` gate_up CTAs with `smem` bytes each can be
// resident at once (occupancy calculator; cached per device and shape).
int gate_up_tc_active_clusters(int cl, int smem, bool mx = false) {
  static std::mutex mu;
  static std::vector<std::array<int, 5>> cache;  // {device, cl, smem, mx, clusters}
  int devno = 0;
  cudaGetDevice(&devno);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& c : cache)
      if (c[0] == devno && c[1] == cl && c[2] == smem && c[3] == (int)mx) return c[4];
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cl);
  cfg.blockDim = dim3(mx ? wdb::TC_MX_THREADS : wdb::TC_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nc = 0;
  // All instantiations of one kernel have the same launch shape and resources.
  const void* fn = mx ? (const void*)wdb::moe_gate_up_tc_mx_kernel<wdb::ROUTE_LARGE>
                      : (const void*)wdb::moe_gate_up_tc_kernel<wdb::ROUTE_LARGE>;
  if (cudaOccupancyMaxActiveClusters(&nc, fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    nc = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({devno, cl, smem, (int)mx, nc});
  return nc;
}

// Tensor-core gate_up for one launch chunk of bn tokens.
int gate_up_tc_launch(const DeviceInfo* dev, const void* x, const void* w, const int32_t* ids,
                      void* out, int bn, int E, int topk, int hidden, int inter,
                      uint32_t* status, cudaStream_t s) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(WD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tm_w, tm_x;
  // w_gate_up [E, 2I, H] viewed as (k, neuron, gate|up, expert): one box is
  // 64 K-columns of 64 gate rows followed by the 64 matching up rows.
  const cuuint64_t wdim[4] = {(cuuint64_t)hidden, (cuuint64_t)inter, 2, (cuuint64_t)E};
  const cuuint64_t wstr[3] = {(cuuint64_t)hidden * 2, (cuuint64_t)inter * hidden * 2,
                              (cuuint64_t)2 * inter * hidden * 2};
  const cuuint32_t wbox[4] = {(cuuint32_t)wdb::TC_BK, (cuuint32_t)wdb::TC_NEUR, 2, 1};
  const cuuint32_t ones[4] = {1, 1, 1, 1};
  CUresult cr = enc(&tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(w), wdim, wstr,
                    wbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    WD_TC_L2PROMO, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (w_gate_up) encode failed");
  const cuuint64_t xdim[2] = {(cuuint64_t)hidden, (cuuint64_t)bn};
  const cuuint64_t xstr[1] = {(cuuint64_t)hidden * 2};
  const int npad = (bn + 15) / 16 * 16;  // MMA N; rows past bn are zero-filled
  const cuuint32_t xbox[2] = {(cuuint32_t)wdb::TC_BK, (cuuint32_t)npad};
  cr = enc(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdim, xstr, xbox,
           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (x) encode failed");

  const int n = bn * topk;
  const int budget = dev->smem_optin - 2048;
  // Stages of WD_TC_KCH 64-wide K chunks (each weight row is then read in
  // WD_TC_KCH * 128 contiguous bytes), as many as fit, at most 8.
  const int kch = WD_TC_KCH;
  auto plan = [&](int cl, int* stages_out) {
    int st = 8;
    while (st > 2 && wdb::gate_up_tc_smem_bytes(st, kch, npad, n, E, cl) > budget) --st;
    *stages_out = st;
    return wdb::gate_up_tc_smem_bytes(st, kch, npad, n, E, cl);
  };
  // Few items (small B): split K over a cluster of cl CTAs, so that the
  // busiest CTA streams ceil(items / clusters) / cl items' worth of weights
  // instead of whole items on a fraction of the SMs.  Items are estimated
  // from the expected number of distinct experts under uniform routing.
  const int n_tiles = (inter + wdb::TC_NEUR - 1) / wdb::TC_NEUR;
  const double u_est =
      E * (1.0 - std::pow(1.0 - std::min(topk, E) / (double)E, (double)bn));
  const int items_est = std::max(1, (int)std::ceil(u_est)) * n_tiles;
  int cl = 1, stages = 0, ncl = 0;
  int smem = plan(1, &stages);
  double best = 1e30;
  const int nkc_all = (hidden + wdb::TC_BK - 1) / wdb::TC_BK;
  for (int c = 1; c <= std::min(WD_TC_MAX_CLUSTER, nkc_all); ++c) {  // >= 1 K chunk per CTA
    int st = 0;
    const int sm = plan(c, &st);
    if (sm > budget) continue;
    int nc = dev->sm_count / c;
    if (c > 1) nc = std::min(nc, gate_up_tc_active_clusters(c, sm));
    if (nc < 1) continue;
    const double cost = std::ceil((double)items_est / nc) / c + 0.02 * (c - 1);
    if (cost < best) { best = cost; cl = c; stages = st; smem = sm; ncl = nc; }
  }
  if (smem > budget) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
  wdb::GateUpTcArgs a;
  a.ids = ids;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.status = status;
  a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
  a.stages = stages;
  a.npad = npad;
  a.kch = kch;
  a.cl = cl;
  a.conv = 0;
  a.xstages = 0;
  const long long work = (long long)n * n_tiles;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if (cl > 1) {
    cfg.gridDim = dim3((unsigned)(ncl * cl));
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  } else {
    cfg.gridDim = dim3((unsigned)std::min<long long>(dev->sm_count, work));
  }
  cfg.blockDim = dim3(wdb::TC_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaError_t err =
      bn * topk <= 64
          ? cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_tc_kernel<wdb::ROUTE_SMALL>, tm_w, tm_x, a)
          : cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_tc_kernel<wdb::ROUTE_LARGE>, tm_w, tm_x, a);
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA, std::string("gate_up (tensor core) launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

// Tensor-core gate_up with MXFP8 weights for one launch chunk of bn <= 16
// tokens: E4M3 boxes of 128 K-bytes x 128 rows and their scale boxes are
// decoded to bf16 on chip by the kernel's converter warps.
int gate_up_tc_mx_launch(const DeviceInfo* dev, const void* x, const uint8_t* w,
                         const uint8_t* wscale, const int32_t* ids, void* out, int bn, int E,
                         int topk, int hidden, int inter, uint32_t* status, cudaStream_t s) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(WD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tm_w, tm_x, tm_s;
  const cuuint32_t ones[4] = {1, 1, 1, 1};
  // E4M3 bytes [E, 2I, H] and scales [E, 2I, H / 32], both viewed as
  // (k, neuron, gate|up, expert); 64 gate rows then the matching up rows.
  const cuuint64_t wdim[4] = {(cuuint64_t)hidden, (cuuint64_t)inter, 2, (cuuint64_t)E};
  const cuuint64_t wstr[3] = {(cuuint64_t)hidden, (cuuint64_t)inter * hidden,
                              (cuuint64_t)2 * inter * hidden};
  const cuuint32_t wbox[4] = {128, (cuuint32_t)wdb::TC_NEUR, 2, 1};
  CUresult cr = enc(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(w), wdim, wstr,
                    wbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    WD_TC_L2PROMO, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (MXFP8 w_gate_up) encode failed");
  const cuuint64_t nb = (cuuint64_t)hidden / 32;
  const cuuint64_t sdim[4] = {nb, (cuuint64_t)inter, 2, (cuuint64_t)E};
  const cuuint64_t sstr[3] = {nb, (cuuint64_t)inter * nb, (cuuint64_t)2 * inter * nb};
  const cuuint32_t sbox[4] = {16, (cuuint32_t)wdb::TC_NEUR, 2, 1};
  cr = enc(&tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(wscale), sdim, sstr, sbox,
           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (MXFP8 scales) encode failed");
  const cuuint64_t xdim[2] = {(cuuint64_t)hidden, (cuuint64_t)bn};
  const cuuint64_t xstr[1] = {(cuuint64_t)hidden * 2};
  const int npad = (bn + 15) / 16 * 16;
  const cuuint32_t xbox[2] = {(cuuint32_t)wdb::TC_BK, (cuuint32_t)npad};
  cr = enc(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdim, xstr, xbox,
           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (x) encode failed");

  const int n = bn * topk;
  const int budget = dev->smem_optin - 2048;
  // Two converted boxes between converters and MMAs; E4M3 stages and x
  // stages in equal numbers (the single producer thread issues both in stage
  // order, so a shallower x ring would hold back the weight stream), as many
  // as fit.
  constexpr int kConv = 2;
  auto plan = [&](int cl, int* stages_out) {
    int st = 6;
    while (st > 2 && wdb::gate_up_tc_mx_smem_bytes(st, st, kConv, npad, n, E, cl) > budget) --st;
    *stages_out = st;
    return wdb::gate_up_tc_mx_smem_bytes(st, st, kConv, npad, n, E, cl);
  };
  // Split K over clusters when items are few (the bf16 kernel's cost model).
  const int n_tiles = (inter + wdb::TC_NEUR - 1) / wdb::TC_NEUR;
  const double u_est =
      E * (1.0 - std::pow(1.0 - std::min(topk, E) / (double)E, (double)bn));
  const int items_est = std::max(1, (int)std::ceil(u_est)) * n_tiles;
  int cl = 1, stages = 0, ncl = 0;
  int smem = plan(1, &stages);
  double best = 1e30;
  const int nks_all = hidden / wdb::TC_MX_STAGE_K;
  for (int c = 1; c <= std::min(WD_TC_MAX_CLUSTER, nks_all); ++c) {  // >= 1 stage per CTA
    int st = 0;
    const int sm = plan(c, &st);
    if (sm > budget) continue;
    int nc = dev->sm_count / c;
    if (c > 1) nc = std::min(nc, gate_up_tc_active_clusters(c, sm, true));
    if (nc < 1) continue;
    const double cost = std::ceil((double)items_est / nc) / c + 0.02 * (c - 1);
    if (cost < best) { best = cost; cl = c; stages = st; smem = sm; ncl = nc; }
  }
  if (smem > budget) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
  wdb::GateUpTcArgs a;
  a.ids = ids;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.status = status;
  a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
  a.stages = stages;
  a.npad = npad;
  a.kch = 0;
  a.cl = cl;
  a.conv = kConv;
  a.xstages = stages;
  const long long work = (long long)n * n_tiles;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if (cl > 1) {
    cfg.gridDim = dim3((unsigned)(ncl * cl));
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  } else {
    cfg.gridDim = dim3((unsigned)std::min<long long>(dev->sm_count, work));
  }
  cfg.blockDim = dim3(wdb::TC_MX_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaError_t err =
      n <= 64
          ? cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_tc_mx_kernel<wdb::ROUTE_SMALL>, tm_w, tm_x,
                               tm_s, a)
          : cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_tc_mx_kernel<wdb::ROUTE_LARGE>, tm_w, tm_x,
                               tm_s, a);
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA,
                std::string("gate_up (MXFP8, tensor core) launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

// Whether a call of B tokens runs on the tensor-core kernel (in launches of
// at most TC_NMAX tokens).
bool gate_up_tc_applies(int B, int E, int hidden) {
  const int p = gate_up_path();
  if (p == 1) return false;
  if (E > wdb::MAX_DEDUP_E || hidden % 8 != 0) return false;
  return p == 2 || B >= WD_TC_MIN_TOKENS;
}

// The same for MXFP8 weights (in launches of at most TC_MX_NMAX tokens).
// The scale rows (hidden / 32 bytes) must be tensor-map strides (16-byte
// multiples), so hidden % 512 == 0.
bool gate_up_tc_mx_applies(int B, int E, int hidden) {
  const int p = gate_up_path();
  if (p == 1) return false;
  if (E > wdb::MAX_DEDUP_E || hidden % 512 != 0) return false;
  return p == 2 || B >= WD_TC_MX_MIN_TOKENS;
}

template <int FMT>
int gate_up_impl(const void* x, const uint8_t* w, const uint8_t* wscale, const int32_t* ids,
                 void* out, int B, int E, int topk, int hidden, int inter, uint32_t* status,
                 void* stream) {
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (FMT == wdb::W_BF16 && hidden % 8 != 0)
    return fail(WD_ERR_SHAPE, "hidden must be a multiple of 8 (16-byte weight rows)");
  if (FMT == wdb::W_E4M3 && hidden % 32 != 0)
    return fail(WD_ERR_SHAPE, "hidden must be a multiple of 32 (MXFP8 block size)");
  if (B == 0) return WD_OK;
  if (!x || !w || !ids || !out || (FMT == wdb::W_E4M3 && !wscale))
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(x) || !aligned16(w) || (FMT == wdb::W_E4M3 && !aligned16(wscale)))
    return fail(WD_ERR_ALIGNMENT, "x and w_gate_up must be 16-byte aligned");
  if (FMT == wdb::W_E4M3 && ((size_t)E * 2 * inter * (hidden / 32)) % 16 != 0)
    return fail(WD_ERR_ALIGNMENT, "MXFP8 scale tensor size must be a multiple of 16 bytes");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;

  constexpr int WB = FMT == wdb::W_BF16 ? 2 : 1;
  const bool tc = FMT == wdb::W_BF16 ? gate_up_tc_applies(B, E, hidden)
                                     : gate_up_tc_mx_applies(B, E, hidden);
  int tb = std::max(1, wdb::MAX_SLOTS / topk);  // tokens per launch
  if (tc) tb = std::min(tb, FMT == wdb::W_BF16 ? wdb::TC_NMAX : wdb::TC_MX_NMAX);
  if ((long long)std::min(tb, B) * topk * inter >= (1LL << 31))
    return fail(WD_ERR_UNSUPPORTED, "B*topk*inter per launch must be < 2^31");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tb) {
    const int bn = std::min(tb, B - b0);
    const int n = bn * topk;
    if (tc) {
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x) + (size_t)b0 * hidden;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)b0 * topk * inter;
      rc = FMT == wdb::W_BF16
               ? gate_up_tc_launch(dev, xb, w, ids + (size_t)b0 * topk, ob, bn, E, topk, hidden,
                                   inter, status, s)
               : gate_up_tc_mx_launch(dev, xb, w, wscale, ids + (size_t)b0 * topk, ob, bn, E,
                                      topk, hidden, inter, status, s);
      if (rc) return rc;
      continue;
    }
    const bool dedup = bn > 1 && E <= wdb::MAX_DEDUP_E;
    // Ring: 8 warps x `depth` slots of (gate, up) row chunks of up to 4 KB
    // each, a chunk never longer than the row (hidden < 4 KB of weights gives
    // smaller slots rather than half-empty ones); x staged in shared memory
    // if it fits in 128 KB.  Preference order: x staged with the deepest ring
    // that fits (up to GU_DEPTH_MAX slots per warp: the bytes in flight per
    // SM set the rate of this latency-bound stream; at B = 1 a CTA's whole
    // share is then requested at once), then 2 KB chunks, then x from L2.
    const long long x_bytes = (long long)bn * hidden * 2;
    const bool x_fits = x_bytes <= 128 * 1024;
    const int kc_full = std::min(4096 / WB, ((hidden + 31) / 32) * 32);
    struct Choice { int kc; bool x_smem; };
    const Choice choices[] = {{kc_full, x_fits}, {std::min(kc_full, 2048 / WB), x_fits},
                              {std::min(kc_full, 2048 / WB), false}};
    int kc = 0, depth = 0, smem = 0;
    bool x_smem = false;
    auto plan = [&](int budget) {
      for (const Choice& c : choices) {
        for (int d = wdb::GU_DEPTH_MAX; d >= 2 && !smem; --d) {
          const int need = wdb::gate_up_smem_bytes(d, wdb::gate_up_stage_bytes(FMT, c.kc),
                                                   c.x_smem ? (int)x_bytes : 0, n, E, dedup);
          if (need <= budget) {
            kc = c.kc; depth = d; x_smem = c.x_smem; smem = need;
          }
        }
        if (smem) return;
      }
    };
    // MXFP8: two CTAs per SM when a plan fits half of the SM's shared memory
    // (the E4M3 decode makes this stream issue-latency bound; twice the warps
    // per scheduler hide it).  bf16 and larger plans: one CTA per SM.
    int ctas_per_sm = 1;
    if (FMT == wdb::W_E4M3) {
      plan(dev->smem_per_sm / 2 - dev->smem_reserved - 1024);
      if (smem) ctas_per_sm = 2;
    }
    if (!smem) plan(dev->smem_optin - 2048);
    if (!smem) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
    wdb::GateUpArgs a;
    a.x = reinterpret_cast<const __nv_bfloat16*>(x) + (size_t)b0 * hidden;
    a.w = w;
    a.wscale = wscale;
    a.ids = ids + (size_t)b0 * topk;
    a.out = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)b0 * topk * inter;
    a.status = status;
    a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
    a.dedup = dedup ? 1 : 0;
    a.kc = kc;
    a.depth = depth;
    a.stage_bytes = wdb::gate_up_stage_bytes(FMT, kc);
    a.x_smem = x_smem ? 1 : 0;
    const long long work = (long long)n * inter;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<long long>((long long)ctas_per_sm * dev->sm_count, work));
    cfg.blockDim = dim3(wdb::GU_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cfg.attrs = nullptr;
    cfg.numAttrs = 0;
    cudaError_t err =
        n <= 64 ? cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_kernel<FMT, wdb::ROUTE_SMALL>, a)
                : cudaLaunchKernelEx(&cfg, wdb::moe_gate_up_kernel<FMT, wdb::ROUTE_LARGE>, a);
    if (err != cudaSuccess)
      return fail(WD_ERR_CUDA, std::string("gate_up launch: ") + cudaGetErrorString(err));
    note_launch();
  }
  return WD_OK;
}

// Largest cluster size CL <= 8 such that the ceil(hidden / 128) row tiles
// times CL CTAs fit on the SMs at once (checked with the occupancy
// calculator for this launch configuration); 0 if none.  Sizes that are not
// powers of two matter for few tiles: at hidden 2048 (16 tiles) clusters of 8
// of the MXFP8 kernel do not all fit, and 7 gives 112 CTAs where 4 gave 64.
int down_tc_cluster(const DeviceInfo* dev, int hidden, int smem, bool mx = false) {
  static std::mutex mu;
  static std::vector<std::array<int, 5>> cache;  // {device, hidden, smem, mx, CL}
  int devno = 0;
  cudaGetDevice(&devno);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& c : cache)
      if (c[0] == devno && c[1] == hidden && c[2] == smem && c[3] == (int)mx) return c[4];
  }
  const int T = (hidden + wdb::DTC_M - 1) / wdb::DTC_M;
  int best = 0;
  for (int cl = 8; cl >= 1; --cl) {
    if (T * cl > dev->sm_count) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(T * cl));
    cfg.blockDim = dim3(mx ? wdb::DTC_MX_THREADS : wdb::DTC_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nc = 0;
    // All instantiations of one kernel have the same launch shape and resources.
    const void* fn = mx ? (const void*)wdb::moe_down_tc_mx_kernel<wdb::ROUTE_LARGE>
                        : (const void*)wdb::moe_down_tc_kernel<false, wdb::ROUTE_LARGE>;
    if (cudaOccupancyMaxActiveClusters(&nc, fn, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (nc >= T) { best = cl; break; }
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({devno, hidden, smem, (int)mx, best});
  return best;
}

bool down_tc_applies(int B, int E, int hidden, int inter, int sms) {
  const int p = down_path();
  if (p == 1) return false;
  if (E > wdb::MAX_DEDUP_E || inter > wdb::DTC_MAXKC * wdb::DTC_BK) return false;
  if ((hidden + wdb::DTC_M - 1) / wdb::DTC_M > sms) return false;
  return p == 2 || B >= WD_DTC_MIN_TOKENS;
}

// MXFP8 weights on the tensor-core down kernel (in launches of at most
// DTC_MX_NMAX tokens): whole 128-K E4M3 boxes (inter % 128 == 0), whole row
// tiles and item scales that are 16-byte-aligned bulk copies (hidden % 128
// == 0, hidden * inter % 512 == 0).
// Automatic from 8 tokens.  Measured (H 2048, I 768, E 128, top-8, cold,
// B200; clusters of 7 over the 16 row tiles), tensor cores vs SIMT: B = 2
// 30.4 vs 32.1 us, B = 4 40.9 vs 38.9, B = 8 65.2 vs 78.0, B = 16 94.2 vs
// 189.9.
#ifndef WD_DTC_MX_MIN_TOKENS
#define WD_DTC_MX_MIN_TOKENS 8
#endif
bool down_tc_mx_applies(int B, int E, int hidden, int inter, int sms) {
  const int p = down_path();
  if (p == 1) return false;
  if (E > wdb::MAX_DEDUP_E || inter > wdb::DTC_MAXKC * wdb::DTC_BK || inter % 128 != 0 ||
      hidden % wdb::DTC_M != 0 || ((long long)hidden * inter) % 512 != 0)
    return false;
  if (hidden / wdb::DTC_M > sms) return false;
  return p == 2 || B >= WD_DTC_MX_MIN_TOKENS;
}

// MXFP8 tensor-core down for one launch chunk of bn <= DTC_MX_NMAX tokens.
int down_tc_mx_launch(const DeviceInfo* dev, const void* h, const uint8_t* w, const uint8_t* wscale,
                      const int32_t* ids, const float* scale, void* out, int out_fp32, int bn,
                      int E, int topk, int hidden, int inter, uint32_t* status, cudaStream_t s) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(WD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  // E4M3 bytes [E, H, I]: box = 128 K-bytes of 128 rows of one expert.
  CUtensorMap tm;
  const cuuint64_t dim[3] = {(cuuint64_t)inter, (cuuint64_t)hidden, (cuuint64_t)E};
  const cuuint64_t str[2] = {(cuuint64_t)inter, (cuuint64_t)hidden * inter};
  const cuuint32_t box[3] = {128, (cuuint32_t)wdb::DTC_M, 1};
  const cuuint32_t ones[3] = {1, 1, 1};
  CUresult cr = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(w), dim, str, box,
                    ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (MXFP8 w_down) encode failed");
  const int n = bn * topk;
  const int budget = dev->smem_optin - 2048;
  constexpr int kConv = 2;
  const int kc = wdb::down_tc_kc(inter);  // even: inter % 128 == 0
  const int sc = std::min(wdb::DTC_SC, kc);
  int stages = 0, nbuf = 0, smem = 0;
  for (int st = 6; st >= 2 && !smem; --st)
    for (int nb : {8, 6, wdb::DTC_GW}) {
      const int need = wdb::down_tc_mx_smem_bytes(st, sc, nb, kConv, inter, bn, n, E);
      if (need <= budget) {
        stages = st; nbuf = nb; smem = need;
        break;
      }
    }
  if (!smem) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
  const int cl = down_tc_cluster(dev, hidden, smem, true);
  if (cl == 0) return fail(WD_ERR_UNSUPPORTED, "no cluster configuration fits");
  wdb::DownTcArgs a;
  a.h = reinterpret_cast<const __nv_bfloat16*>(h);
  a.ids = ids;
  a.scale = scale;
  a.out = out;
  a.out_fp32 = out_fp32 ? 1 : 0;
  a.status = status;
  a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
  a.stages = stages;
  a.sc = sc;
  a.nbuf = nbuf;
  a.cl = cl;
  a.tp = {};
  a.wscale = wscale;
  a.conv = kConv;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (cl > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)cl;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((hidden / wdb::DTC_M) * cl));
  cfg.blockDim = dim3(wdb::DTC_MX_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t err =
      n <= 64 ? cudaLaunchKernelEx(&cfg, wdb::moe_down_tc_mx_kernel<wdb::ROUTE_SMALL>, tm, a)
              : cudaLaunchKernelEx(&cfg, wdb::moe_down_tc_mx_kernel<wdb::ROUTE_LARGE>, tm, a);
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA,
                std::string("down (MXFP8, tensor core) launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

// Tensor-core down for one launch chunk of bn tokens; returns WD_ERR_UNSUPPORTED
// (nothing launched) if no cluster configuration fits, so the caller can
// fall back to the SIMT kernel.
int down_tc_launch(const DeviceInfo* dev, const void* h, const void* w, const int32_t* ids,
                   const float* scale, void* out, int out_fp32, int bn, int E, int topk,
                   int hidden, int inter, uint32_t* status, cudaStream_t s,
                   const wdb::TpArgs* tp = nullptr) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(WD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  // w_down [E, H, I]: box = 64 K-columns of 128 rows of one expert.
  CUtensorMap tm;
  const cuuint64_t dim[3] = {(cuuint64_t)inter, (cuuint64_t)hidden, (cuuint64_t)E};
  const cuuint64_t str[2] = {(cuuint64_t)inter * 2, (cuuint64_t)hidden * inter * 2};
  const cuuint32_t box[3] = {(cuuint32_t)wdb::DTC_BK, (cuuint32_t)wdb::DTC_M, 1};
  const cuuint32_t ones[3] = {1, 1, 1};
  CUresult cr = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w), dim, str, box,
                    ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (w_down) encode failed");
  const int n = bn * topk;
  const int budget = dev->smem_optin - 2048;
  // Weight ring: as many K chunks in flight as fit (stages x chunks per
  // stage), never fewer h slices than gather warps.
  const int kc = wdb::down_tc_kc(inter);
  int stages = 0, sc = 0, nbuf = 0, smem = 0;
  for (int c : {wdb::DTC_SC, 2, 1}) {
    const int scc = std::min(c, kc);
    for (int st = 6; st >= 2 && !smem; --st)
      for (int nb : {8, 6, wdb::DTC_GW}) {
        const int need = wdb::down_tc_smem_bytes(st, scc, nb, inter, bn, n, E);
        if (need <= budget) {
          stages = st; sc = scc; nbuf = nb; smem = need;
          break;
        }
      }
    if (smem) break;
  }
  if (!smem) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
  const int cl = down_tc_cluster(dev, hidden, smem);
  if (cl == 0) return fail(WD_ERR_UNSUPPORTED, "no cluster configuration fits");
  wdb::DownTcArgs a;
  a.h = reinterpret_cast<const __nv_bfloat16*>(h);
  a.ids = ids;
  a.scale = scale;
  a.out = out;
  a.out_fp32 = out_fp32 ? 1 : 0;
  a.status = status;
  a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
  a.stages = stages;
  a.sc = sc;
  a.nbuf = nbuf;
  a.cl = cl;
  a.tp = {};
  a.wscale = nullptr;
  a.conv = 0;
  if (tp) {
    if (((hidden + wdb::DTC_M - 1) / wdb::DTC_M) * cl > tp->max_ctas)
      return fail(WD_ERR_UNSUPPORTED, "grid larger than the communicator's epoch array");
    a.tp = *tp;
  }
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cl > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)cl;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((hidden + wdb::DTC_M - 1) / wdb::DTC_M) * cl));
  cfg.blockDim = dim3(wdb::DTC_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t err =
      a.tp.world > 1 ? cudaLaunchKernelEx(&cfg, wdb::moe_down_tc_kernel<true, wdb::ROUTE_ANY>, tm, a)
      : n <= 64      ? cudaLaunchKernelEx(&cfg, wdb::moe_down_tc_kernel<false, wdb::ROUTE_SMALL>, tm, a)
                     : cudaLaunchKernelEx(&cfg, wdb::moe_down_tc_kernel<false, wdb::ROUTE_LARGE>, tm, a);
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA, std::string("down (tensor core) launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

template <int FMT>
int down_impl(const void* h, const uint8_t* w, const uint8_t* wscale, const int32_t* ids,
              const float* scale, void* out, int out_fp32, int B, int E, int topk, int hidden,
              int inter, uint32_t* status, void* stream) {
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (FMT == wdb::W_BF16 && inter % 8 != 0)
    return fail(WD_ERR_SHAPE, "inter must be a multiple of 8 (16-byte weight rows)");
  if (FMT == wdb::W_E4M3 && inter % 32 != 0)
    return fail(WD_ERR_SHAPE, "inter must be a multiple of 32 (MXFP8 block size)");
  if (B == 0) return WD_OK;
  if (!h || !w || !ids || !scale || !out || (FMT == wdb::W_E4M3 && !wscale))
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(h) || !aligned16(w) || (FMT == wdb::W_E4M3 && !aligned16(wscale)))
    return fail(WD_ERR_ALIGNMENT, "h and w_down must be 16-byte aligned");
  if (FMT == wdb::W_E4M3 && ((size_t)E * hidden * (inter / 32)) % 16 != 0)
    return fail(WD_ERR_ALIGNMENT, "MXFP8 scale tensor size must be a multiple of 16 bytes");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;

  constexpr int WB = FMT == wdb::W_BF16 ? 2 : 1;
  constexpr int EPV = FMT == wdb::W_BF16 ? 8 : 16;
  const int row_bytes = inter * WB;
  const int nvec = inter / EPV;
  const int lpr = nvec <= 32 ? 8 : (nvec <= 64 ? 16 : 32);
  int grid = 0, rows_max = 0, rows_chunk = 0, stage_bytes = 0, depth = 0, tb = 0;
  // Geometry for a grid of g CTAs, each owning a block of rows_max rows.
  auto geometry = [&](int g) {
    grid = g;
    rows_max = (hidden + grid - 1) / grid;
    // Item = chunk of >= 4 KB of contiguous rows (smaller bulk copies do not
    // saturate HBM), chunks of one CTA's block as even as that allows.
    const int rc_min = std::min(rows_max, std::max(1, (4096 + row_bytes - 1) / row_bytes));
    const int nch = std::max(1, rows_max / rc_min);
    rows_chunk = (rows_max + nch - 1) / nch;
    stage_bytes = rows_chunk * row_bytes + wdb::down_scale_area<FMT>(rows_chunk, inter);
    stage_bytes = ((stage_bytes + 127) / 128) * 128;
    depth = std::min(4, std::max(2, (96 * 1024) / (wdb::NWARPS * stage_bytes)));
    // Tokens per launch: routing capacity and the 8 per-warp FP32 tiles.
    tb = std::max(1, wdb::MAX_SLOTS / topk);
    tb = std::min(tb, std::max(1, (64 * 1024) / (4 * wdb::NWARPS * rows_max)));
  };
  auto smem_need = [&](int bn, bool h_smem) {
    const int n = bn * topk;
    const bool dedup = bn > 1 && E <= wdb::MAX_DEDUP_E;
    return wdb::down_smem_bytes(depth, stage_bytes, h_smem ? n * inter * 2 : 0, bn, rows_max, n,
                                E, dedup);
  };
  // MXFP8: two CTAs per SM when every launch of the call fits half of the
  // SM's shared memory (the E4M3 decode makes this stream issue-latency
  // bound; twice the warps per scheduler hide it).  bf16: one CTA per SM.
  int budget = dev->smem_optin - 2048;
  if (FMT == wdb::W_E4M3 && hidden / 4 >= 2 * dev->sm_count) {
    geometry(2 * dev->sm_count);
    const int half = dev->smem_per_sm / 2 - dev->smem_reserved - 1024;
    if (smem_need(std::min(tb, B), false) <= half)
      budget = half;
    else
      grid = 0;
  }
  if (!grid) geometry(std::max(1, std::min(dev->sm_count, hidden / 4)));
  const bool tc = FMT == wdb::W_BF16 ? down_tc_applies(B, E, hidden, inter, dev->sm_count)
                                     : down_tc_mx_applies(B, E, hidden, inter, dev->sm_count);
  if (tc)
    tb = std::min(std::max(1, wdb::MAX_SLOTS / topk),
                  FMT == wdb::W_BF16 ? 64 : wdb::DTC_MX_NMAX);

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t out_elem = out_fp32 ? 4 : 2;
  for (int b0 = 0; b0 < B; b0 += tb) {
    const int bn = std::min(tb, B - b0);
    const int n = bn * topk;
    if (tc) {
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(h) + (size_t)b0 * topk * inter;
      uint8_t* ob = reinterpret_cast<uint8_t*>(out) + (size_t)b0 * hidden * out_elem;
      rc = FMT == wdb::W_BF16
               ? down_tc_launch(dev, hb, w, ids + (size_t)b0 * topk, scale + (size_t)b0 * topk, ob,
                                out_fp32, bn, E, topk, hidden, inter, status, s)
               : down_tc_mx_launch(dev, hb, w, wscale, ids + (size_t)b0 * topk,
                                   scale + (size_t)b0 * topk, ob, out_fp32, bn, E, topk, hidden,
                                   inter, status, s);
      if (rc) return rc;
      continue;
    }
    const bool dedup = bn > 1 && E <= wdb::MAX_DEDUP_E;
    const long long h_bytes = (long long)n * inter * 2;
    bool h_smem = h_bytes <= 64 * 1024;
    if (smem_need(bn, h_smem) > budget) h_smem = false;
    const int smem = smem_need(bn, h_smem);
    if (smem > budget) return fail(WD_ERR_UNSUPPORTED, "shared memory budget exceeded");
    wdb::DownArgs a;
    a.h = reinterpret_cast<const __nv_bfloat16*>(h) + (size_t)b0 * topk * inter;
    a.w = w;
    a.wscale = wscale;
    a.ids = ids + (size_t)b0 * topk;
    a.scale = scale + (size_t)b0 * topk;
    a.out = reinterpret_cast<uint8_t*>(out) + (size_t)b0 * hidden * out_elem;
    a.out_fp32 = out_fp32 ? 1 : 0;
    a.status = status;
    a.B = bn; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
    a.dedup = dedup ? 1 : 0;
    a.depth = depth;
    a.rc = rows_chunk;
    a.lpr = lpr;
    a.stage_bytes = stage_bytes;
    a.rows_max = rows_max;
    a.h_smem = h_smem ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(wdb::DN_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t err =
        n <= 64 ? cudaLaunchKernelEx(&cfg, wdb::moe_down_kernel<FMT, wdb::ROUTE_SMALL>, a)
                : cudaLaunchKernelEx(&cfg, wdb::moe_down_kernel<FMT, wdb::ROUTE_LARGE>, a);
    if (err != cudaSuccess)
      return fail(WD_ERR_CUDA, std::string("down launch: ") + cudaGetErrorString(err));
    note_launch();
  }
  return WD_OK;
}

// ---- single-launch FFN ------------------------------------------------------
struct FfnPlan {
  int nw = 0;  // warps per CTA (block size / 32)
  int depth = 0, kc = 0, rc = 0, rows_max = 0, stage_bytes = 0, xh_bytes = 0;
  int smem = 0, grid = 0;
  bool dedup = false;
};

// Whether moe_ffn_kernel runs on this device with `smem` bytes of shared
// memory and nw warps at one CTA per SM (cooperative launch: all CTAs
// co-resident).
bool ffn_fits(const DeviceInfo* dev, int smem, int nw) {
  static std::mutex mu;
  static std::vector<std::array<int, 4>> cache;  // {device, smem, nw, fits}
  int devno = 0;
  cudaGetDevice(&devno);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& c : cache)
      if (c[0] == devno && c[1] == smem && c[2] == nw) return c[3] != 0;
  }
  int nb = 0;
  // both instantiations: the same registers and shared memory
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, wdb::moe_ffn_kernel<true>, nw * 32,
                                                    (size_t)smem) != cudaSuccess) {
    cudaGetLastError();
    nb = 0;
  }
  (void)dev;
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({devno, smem, nw, nb >= 1 ? 1 : 0});
  return nb >= 1;
}

// Routed slots up to which the automatic choice takes the single launch.
// Measured on B200 (H 4096, I 192, top-8, cold L2): 22.6 / 30.6 / 43.0 us at
// B = 1 / 2 / 4 against 30.9 / 36.5 / 49.2 us for the two kernels; at B = 8
// the two kernels (tensor-core down) are as fast (66.7 vs 67.7 us).
#ifndef WD_FFN_AUTO_MAX_SLOTS
#define WD_FFN_AUTO_MAX_SLOTS 32
#endif

// Routed slots from which the automatic choice takes the tensor-core single
// launch (moe_ffn_tc_kernel) where it applies.  Measured on B200 (H 4096,
// I 192, E 128, top-8, cold L2, us): B = 8 63.0 vs 61.8 as SIMT gate_up +
// tensor-core down; B = 16 86.2 vs 91.8; B = 32 114.6 / 111.9 vs 112.7 (two
// runs); B = 64 123.4 vs 129.1 as the two tensor-core kernels.
#ifndef WD_FFN_TC_MIN_SLOTS
#define WD_FFN_TC_MIN_SLOTS 65
#endif

// Launch geometry of the single-launch FFN, or false where it does not apply:
// more than max_slots routed slots (at most 64), E above the dedup table, or
// x / h of the call too large for shared memory next to a two-slot ring.
bool ffn_plan(const DeviceInfo* dev, int B, int E, int topk, int hidden, int inter, int max_slots,
              FfnPlan* pl) {
  const int n = B * topk;
  if (n < 1 || n > std::min(max_slots, wdb::FFN_MAX_SLOTS)) return false;
  if (hidden % 8 != 0 || inter % 8 != 0) return false;
  const bool dedup = n > 1;
  if (dedup && E > wdb::MAX_DEDUP_E) return false;
  FfnPlan p;
  p.grid = dev->sm_count;
  p.rows_max = (hidden + p.grid - 1) / p.grid;
  p.kc = 2048;  // bf16 elements: 4 KB gate and up row chunks
  const int row_bytes = inter * 2;
  p.stage_bytes = std::max(wdb::gate_up_stage_bytes(wdb::W_BF16, p.kc), ((row_bytes + 127) / 128) * 128);
  // Down chunks: as many of the CTA's rows as fit a slot, split evenly.  With
  // fewer than 4 rows per slot (inter > 1024) the down phase becomes a long
  // run of tiny stages per warp: measured slower than the two kernels
  // (inter 1536, B = 1: 112 vs 78 us), so the single launch stops there.
  const int rc_cap = std::max(1, p.stage_bytes / row_bytes);
  if (rc_cap < 4 && p.rows_max > rc_cap) return false;
  const int nch = (p.rows_max + rc_cap - 1) / rc_cap;
  p.rc = (p.rows_max + nch - 1) / nch;
  // Automatic choice: at most ~8 down stages per warp (slots x chunks per
  // group / 8 warps).  Measured crossover: H 2048, inter 768, B = 4 (96
  // stages per CTA) ran 79.8 us as one launch vs 75.9 us as two kernels,
  // while H 4096, inter 192, B = 4 (64) gained 6 us.
  if (max_slots < wdb::FFN_MAX_SLOTS && n * nch > 64) return false;
  p.xh_bytes = std::max(B * hidden * 2, n * inter * 2);
  p.dedup = dedup;
  // The most warps that fit (each with a ring of at least two slots), then
  // the deepest ring for them (kernel comment in wd_ffn.cuh: measured).
  const int budget = dev->smem_optin - 2048;
  for (int nw = wdb::FFN_MAX_WARPS; nw >= 4; --nw) {
    for (int depth : {4, 3, 2}) {
      const int need = wdb::ffn_smem_bytes(nw, depth, p.stage_bytes, p.xh_bytes, B, p.rows_max,
                                           n, E, dedup);
      if (need <= budget && ffn_fits(dev, need, nw)) {
        p.nw = nw;
        p.depth = depth;
        p.smem = need;
        *pl = p;
        return true;
      }
    }
  }
  return false;
}

int ffn_launch(const DeviceInfo* dev, const FfnPlan& p, const void* x, const void* w_gu,
               const void* w_dn, const int32_t* ids, const float* scale, void* h, uint32_t* sync,
               void* y, int out_fp32, int B, int E, int topk, int hidden, int inter,
               uint32_t* status, cudaStream_t s, const wdb::TpArgs* tp = nullptr) {
  wdb::FfnArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x);
  a.wgu = reinterpret_cast<const uint8_t*>(w_gu);
  a.wdn = reinterpret_cast<const uint8_t*>(w_dn);
  a.ids = ids;
  a.scale = scale;
  a.h = reinterpret_cast<__nv_bfloat16*>(h);
  a.sync = reinterpret_cast<unsigned long long*>(sync);
  a.out = y;
  a.out_fp32 = out_fp32 ? 1 : 0;
  a.status = status;
  a.B = B; a.E = E; a.K = topk; a.H = hidden; a.I = inter;
  a.dedup = p.dedup ? 1 : 0;
  a.depth = p.depth;
  a.stage_bytes = p.stage_bytes;
  a.kc = p.kc;
  a.rc = p.rc;
  a.rows_max = p.rows_max;
  a.xh_bytes = p.xh_bytes;
  a.tp = {};
  if (tp) a.tp = *tp;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3((unsigned)(p.nw * 32));
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = tp ? cudaLaunchKernelEx(&cfg, wdb::moe_ffn_kernel<true>, a)
                       : cudaLaunchKernelEx(&cfg, wdb::moe_ffn_kernel<false>, a);
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA, std::string("ffn launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

// ---- single-launch FFN on the tensor cores ----------------------------------
struct FfnTcPlan {
  int smem = 0, cl = 0, tiles = 0, npad = 0, route_bytes = 0;
  int gu_stages = 0, kch = 0, gu_cl = 1;
  int dn_stages = 0, dn_sc = 0, dn_nb = 0;
};

// The automatic choice takes it from WD_FFN_TC_MIN_SLOTS routed slots and
// only where its grid is near the SM count and the down items are
// one weight stage (inter <= 256).  Measured against the two kernels (cold,
// us): H 7168 (56 tiles x clusters of 2 = 112 CTAs), I 256, B = 32: 207.2 vs
// 190.5; H 2048, I 768, B = 16: 309.5 vs 195; H 4096, I 1536, B = 16 / 64:
// 538.6 / 751.5 vs 508.0 / 728.7.
bool ffn_tc_auto(const FfnTcPlan& p, int B, int topk, int inter) {
  return B * topk >= WD_FFN_TC_MIN_SLOTS && inter <= 256 && p.tiles * p.cl >= 120;
}

// Largest cluster size cl <= 8 such that the tiles x cl CTAs of
// moe_ffn_tc_kernel with `smem` bytes are all resident at once (the grid
// barrier needs them co-resident); 0 if none.  Cached per device and smem.
int ffn_tc_cluster(const DeviceInfo* dev, int tiles, int smem) {
  static std::mutex mu;
  static std::vector<std::array<int, 4>> cache;  // {device, tiles, smem, cl}
  int devno = 0;
  cudaGetDevice(&devno);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& c : cache)
      if (c[0] == devno && c[1] == tiles && c[2] == smem) return c[3];
  }
  int best = 0;
  for (int cl = 8; cl >= 2 && !best; --cl) {
    if (tiles * cl > dev->sm_count) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles * cl));
    cfg.blockDim = dim3(wdb::DTC_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, wdb::moe_ffn_tc_kernel<wdb::ROUTE_LARGE>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (nc >= tiles) best = cl;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({devno, tiles, smem, best});
  return best;
}

// Launch geometry of moe_ffn_tc_kernel, or false where it does not apply:
// one launch of at most TC_NMAX tokens and MAX_SLOTS routed slots, the
// shapes of both tensor-core kernels, both phases' rings next to the routing
// region in shared memory, and every CTA resident at once.
bool ffn_tc_plan(const DeviceInfo* dev, int B, int E, int topk, int hidden, int inter,
                 FfnTcPlan* out) {
  const int n = B * topk;
  if (B < 1 || B > wdb::TC_NMAX || n > wdb::MAX_SLOTS) return false;
  if (E > wdb::MAX_DEDUP_E || hidden % 8 != 0 || inter % 8 != 0) return false;
  if (inter > wdb::DTC_MAXKC * wdb::DTC_BK) return false;
  FfnTcPlan p;
  p.tiles = (hidden + wdb::DTC_M - 1) / wdb::DTC_M;
  p.npad = (B + 15) / 16 * 16;
  p.kch = WD_TC_KCH;
  p.route_bytes = wdb::ffn_tc_route_bytes(n, E);
  const int route = wdb::route_smem_bytes(n, E, true);
  const int budget = dev->smem_optin - 2048 - p.route_bytes;
  auto gu_plan = [&](int cl, int* stages) {
    for (int st = 8; st >= 2; --st) {
      const int need = wdb::gate_up_tc_smem_bytes(st, p.kch, p.npad, n, E, cl) - route;
      if (need <= budget) { *stages = st; return need; }
    }
    return 0;
  };
  int gu = gu_plan(1, &p.gu_stages);
  if (!gu) return false;
  const int kc = wdb::down_tc_kc(inter);
  int dn = 0;
  for (int c : {wdb::DTC_SC, 2, 1}) {
    const int scc = std::min(c, kc);
    for (int st = 6; st >= 2 && !dn; --st)
      for (int nb : {8, 6, wdb::DTC_GW}) {
        const int need = wdb::down_tc_smem_bytes(st, scc, nb, inter, B, n, E) - route;
        if (need <= budget) {
          dn = need; p.dn_stages = st; p.dn_sc = scc; p.dn_nb = nb;
          break;
        }
      }
    if (dn) break;
  }
  if (!dn) return false;
  p.smem = 1024 + p.route_bytes + std::max(gu, dn);
  if (p.smem > dev->smem_optin - 1024) return false;
  p.cl = ffn_tc_cluster(dev, p.tiles, p.smem);
  if (p.cl == 0) return false;
  // The gate_up phase splits K over the launch's clusters when that lowers
  // the busiest CTA's share: whole items on tiles x cl CTAs, against
  // ceil(items / clusters) / cl (items estimated from the expected distinct
  // experts under uniform routing).  Measured (H 4096, I 192, E 128, top-8):
  // at B = 8 (about 150 items on 128 CTAs) whole items left most CTAs idle
  // while a quarter streamed a second item.
  const int n_tiles = (inter + wdb::TC_NEUR - 1) / wdb::TC_NEUR;
  const double u_est = E * (1.0 - std::pow(1.0 - std::min(topk, E) / (double)E, (double)B));
  const int items = std::max(1, (int)std::ceil(u_est)) * n_tiles;
  const int ctas = p.tiles * p.cl;
  const double cost1 = std::ceil((double)items / ctas);
  const double costc = std::ceil((double)items / p.tiles) / p.cl + 0.02 * (p.cl - 1);
  int st_c = 0;
  const int gu_c = costc < cost1 ? gu_plan(p.cl, &st_c) : 0;
  if (gu_c) {
    const int smem_c = 1024 + p.route_bytes + std::max(gu_c, dn);
    if (smem_c <= dev->smem_optin - 1024 && ffn_tc_cluster(dev, p.tiles, smem_c) == p.cl) {
      p.gu_cl = p.cl;
      p.gu_stages = st_c;
      p.smem = smem_c;
    }
  }
  *out = p;
  return true;
}

// One cooperative launch of moe_ffn_tc_kernel (clusters of p.cl).  Returns
// WD_ERR_UNSUPPORTED, with nothing launched, if the runtime refuses the
// cooperative cluster launch, so the caller can take the two kernels.
int ffn_tc_launch(const DeviceInfo* dev, const FfnTcPlan& p, const void* x, const void* w_gu,
                  const void* w_dn, const int32_t* ids, const float* scale, void* h,
                  unsigned long long* sync, void* y, int out_fp32, int B, int E, int topk,
                  int hidden, int inter, uint32_t* status, cudaStream_t s,
                  const wdb::TpArgs* tp = nullptr) {
  (void)dev;
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(WD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t ones[4] = {1, 1, 1, 1};
  // gate_up weights as (k, neuron, gate|up, expert), boxes of 64 K x 64 gate
  // + 64 up rows; x boxes of 64 K x npad tokens (as gate_up_tc_launch).
  CUtensorMap tm_gw, tm_x, tm_dw;
  const cuuint64_t wdim[4] = {(cuuint64_t)hidden, (cuuint64_t)inter, 2, (cuuint64_t)E};
  const cuuint64_t wstr[3] = {(cuuint64_t)hidden * 2, (cuuint64_t)inter * hidden * 2,
                              (cuuint64_t)2 * inter * hidden * 2};
  const cuuint32_t wbox[4] = {(cuuint32_t)wdb::TC_BK, (cuuint32_t)wdb::TC_NEUR, 2, 1};
  CUresult cr = enc(&tm_gw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(w_gu), wdim,
                    wstr, wbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    WD_TC_L2PROMO, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (w_gate_up) encode failed");
  const cuuint64_t xdim[2] = {(cuuint64_t)hidden, (cuuint64_t)B};
  const cuuint64_t xstr[1] = {(cuuint64_t)hidden * 2};
  const cuuint32_t xbox[2] = {(cuuint32_t)wdb::TC_BK, (cuuint32_t)p.npad};
  cr = enc(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdim, xstr, xbox,
           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (x) encode failed");
  // down weights [E, H, I]: boxes of 64 K x 128 rows of one expert.
  const cuuint64_t ddim[3] = {(cuuint64_t)inter, (cuuint64_t)hidden, (cuuint64_t)E};
  const cuuint64_t dstr[2] = {(cuuint64_t)inter * 2, (cuuint64_t)hidden * inter * 2};
  const cuuint32_t dbox[3] = {(cuuint32_t)wdb::DTC_BK, (cuuint32_t)wdb::DTC_M, 1};
  cr = enc(&tm_dw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w_dn), ddim, dstr, dbox,
           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(WD_ERR_CUDA, "tensor map (w_down) encode failed");

  wdb::FfnTcArgs a = {};
  a.gu.ids = ids;
  a.gu.out = reinterpret_cast<__nv_bfloat16*>(h);
  a.gu.status = status;
  a.gu.B = B; a.gu.E = E; a.gu.K = topk; a.gu.H = hidden; a.gu.I = inter;
  a.gu.stages = p.gu_stages;
  a.gu.npad = p.npad;
  a.gu.kch = p.kch;
  a.gu.cl = p.gu_cl;
  a.gu.conv = 0;
  a.gu.xstages = 0;
  a.dn.h = reinterpret_cast<const __nv_bfloat16*>(h);
  a.dn.ids = ids;
  a.dn.scale = scale;
  a.dn.out = y;
  a.dn.out_fp32 = out_fp32 ? 1 : 0;
  a.dn.status = status;
  a.dn.B = B; a.dn.E = E; a.dn.K = topk; a.dn.H = hidden; a.dn.I = inter;
  a.dn.stages = p.dn_stages;
  a.dn.sc = p.dn_sc;
  a.dn.nbuf = p.dn_nb;
  a.dn.cl = p.cl;
  a.dn.tp = {};
  if (tp) {
    if (p.tiles * p.cl > tp->max_ctas)
      return fail(WD_ERR_UNSUPPORTED, "grid larger than the communicator's epoch array");
    a.dn.tp = *tp;
  }
  a.dn.wscale = nullptr;
  a.dn.conv = 0;
  a.ids = ids;
  a.scale = scale;
  a.sync = sync;
  a.B = B; a.E = E; a.K = topk;
  a.route_bytes = p.route_bytes;

  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.tiles * p.cl));
  cfg.blockDim = dim3(wdb::DTC_THREADS);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err =
      tp          ? cudaLaunchKernelEx(&cfg, wdb::moe_ffn_tc_kernel<wdb::ROUTE_ANY, true>, tm_gw,
                                       tm_x, tm_dw, a)
      : B * topk <= 64
          ? cudaLaunchKernelEx(&cfg, wdb::moe_ffn_tc_kernel<wdb::ROUTE_SMALL>, tm_gw, tm_x, tm_dw, a)
          : cudaLaunchKernelEx(&cfg, wdb::moe_ffn_tc_kernel<wdb::ROUTE_LARGE>, tm_gw, tm_x, tm_dw, a);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(WD_ERR_UNSUPPORTED, std::string("ffn (tensor core) launch: ") +
                                        cudaGetErrorString(err));
  }
  note_launch();
  return WD_OK;
}

// ---- tensor-parallel communicator for the fused all-reduce ------------------
struct TpComm {
  int device = -1;
  int world = 0, rank = 0, max_tokens = 0, hidden = 0, max_ctas = 0;
  int exchange = 0;               // 0 = by size, 1 = one-shot, 2 = two-shot
  void* block = nullptr;          // [2][world][max_tokens][hidden] 8-byte packets
  size_t recv_bytes = 0;
  uint32_t* epochs = nullptr;     // [max_ctas], local only
  void* peer[wdb::TP_MAX_WORLD] = {};  // opened IPC mappings (nullptr for self)
};

// Bytes a rank sends one-shot (B x hidden x 8 x (world - 1)) above which the
// automatic choice takes the two-shot exchange (from four ranks up), which
// sends about 2 / world of that at the price of a second NVLink latency and
// of the owners' wait for every rank.  Measured on four B200s (H 4096,
// I 192 per rank, cold us; one-shot vs two-shot): B = 8 78.5 vs 86.3,
// B = 16 100.9 vs 108.6, B = 32 132.8 vs 144.2, B = 64 (6 MiB sent
// one-shot) 151.2 vs 168.3; on eight, B = 64 (14.7 MiB) 158.8 vs 170.4 --
// the one-shot exchange costs about the same from 0.25 to 15 MiB, so
// two-shot is kept for larger transfers only.
// WARP_DECODE_TP_TWO_SHOT_BYTES overrides it.
size_t tp_two_shot_bytes() {
  static const size_t v = [] {
    const char* e = std::getenv("WARP_DECODE_TP_TWO_SHOT_BYTES");
    return e && *e ? (size_t)std::strtoull(e, nullptr, 10) : (size_t)(16u << 20);
  }();
  return v;
}

wdb::TpArgs make_tp_args(const TpComm* c, int B) {
  wdb::TpArgs tp = {};
  tp.world = c->world;
  tp.rank = c->rank;
  tp.max_tokens = c->max_tokens;
  tp.max_ctas = c->max_ctas;
  tp.epochs = c->epochs;
  // By size: two ranks send as many bytes two-shot as one-shot, so two-shot
  // only from four ranks up.
  const size_t one_shot = (size_t)B * c->hidden * 8 * (c->world - 1);
  tp.two_shot = c->exchange == 2 ||
                (c->exchange == 0 && c->world >= 4 && one_shot > tp_two_shot_bytes()) ? 1 : 0;
  for (int r = 0; r < c->world; ++r)
    tp.recv[r] = static_cast<unsigned long long*>(r == c->rank ? c->block : c->peer[r]);
  return tp;
}

// Device-visible address of `p` for the current device: device (or managed)
// memory of this device as is, page-locked host memory through its mapping.
// Pageable host memory and other devices' memory are refused before anything
// is launched, so the copy kernel only ever dereferences mapped addresses.
int device_view(const void* p, int dev, const char* what, unsigned char** out) {
  cudaPointerAttributes at{};
  const cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(WD_ERR_CUDA, std::string(what) + ": cudaPointerGetAttributes: " + cudaGetErrorString(e));
  }
  switch (at.type) {
    case cudaMemoryTypeHost:
      if (!at.devicePointer)
        return fail(WD_ERR_UNSUPPORTED, std::string(what) + ": page-locked host memory without a device mapping");
      *out = static_cast<unsigned char*>(at.devicePointer);
      return WD_OK;
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      if (at.device != dev)
        return fail(WD_ERR_UNSUPPORTED, std::string(what) + ": memory of another device");
      *out = static_cast<unsigned char*>(const_cast<void*>(p));
      return WD_OK;
    default:
      return fail(WD_ERR_UNSUPPORTED, std::string(what) +
                                          ": pageable host memory (the GPU cannot read or write it; "
                                          "allocate it page-locked or register it)");
  }
}

}  // namespace

extern "C" {

int wd_version(void) { return 100; }

unsigned long long wd_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* wd_error_string(int err) {
  switch (err) {
    case WD_OK: return "ok";
    case WD_ERR_NULL_POINTER: return "null pointer";
    case WD_ERR_SHAPE: return "invalid shape";
    case WD_ERR_ALIGNMENT: return "misaligned pointer";
    case WD_ERR_UNSUPPORTED: return "unsupported shape";
    case WD_ERR_CUDA: return "CUDA error";
    default: return "unknown error";
  }
}

const char* wd_last_error_message(void) { return g_last_error.c_str(); }

int wd_moe_gate_up_3d_batched(const void* x, const void* w_gate_up, const int32_t* topk_ids,
                              void* h_out, int B, int E, int topk, int hidden, int inter,
                              uint32_t* status, void* stream) {
  g_last_error.clear();
  return gate_up_impl<wdb::W_BF16>(x, reinterpret_cast<const uint8_t*>(w_gate_up), nullptr,
                                   topk_ids, h_out, B, E, topk, hidden, inter, status, stream);
}

int wd_moe_down_3d_batched(const void* h, const void* w_down, const int32_t* topk_ids,
                           const float* topk_scale, void* y_out, int out_fp32, int B, int E,
                           int topk, int hidden, int inter, uint32_t* status, void* stream) {
  g_last_error.clear();
  return down_impl<wdb::W_BF16>(h, reinterpret_cast<const uint8_t*>(w_down), nullptr, topk_ids,
                                topk_scale, y_out, out_fp32, B, E, topk, hidden, inter, status,
                                stream);
}

int wd_moe_gate_up_3d_batched_mxfp8(const void* x, const uint8_t* w_q, const uint8_t* w_scale,
                                    const int32_t* topk_ids, void* h_out, int B, int E, int topk,
                                    int hidden, int inter, uint32_t* status, void* stream) {
  g_last_error.clear();
  return gate_up_impl<wdb::W_E4M3>(x, w_q, w_scale, topk_ids, h_out, B, E, topk, hidden, inter,
                                   status, stream);
}

int wd_moe_down_3d_batched_mxfp8(const void* h, const uint8_t* w_q, const uint8_t* w_scale,
                                 const int32_t* topk_ids, const float* topk_scale, void* y_out,
                                 int out_fp32, int B, int E, int topk, int hidden, int inter,
                                 uint32_t* status, void* stream) {
  g_last_error.clear();
  return down_impl<wdb::W_E4M3>(h, w_q, w_scale, topk_ids, topk_scale, y_out, out_fp32, B, E,
                                topk, hidden, inter, status, stream);
}

int wd_set_gate_up_path(int path) {
  g_last_error.clear();
  if (path < 0 || path > 2) return fail(WD_ERR_SHAPE, "path must be 0 (auto), 1 (simt) or 2 (tc)");
  g_gate_up_path.store(path);
  return WD_OK;
}

int wd_set_down_path(int path) {
  g_last_error.clear();
  if (path < 0 || path > 2) return fail(WD_ERR_SHAPE, "path must be 0 (auto), 1 (simt) or 2 (tc)");
  g_down_path.store(path);
  return WD_OK;
}

int wd_moe_router_topk(const void* logits, int logits_fp32, int32_t* topk_ids,
                       float* topk_weights, int B, int E, int topk, int renormalize,
                       void* stream) {
  g_last_error.clear();
  if (B < 0) return fail(WD_ERR_SHAPE, "B must be >= 0");
  if (E < 1 || topk < 1 || topk > E) return fail(WD_ERR_SHAPE, "need 1 <= topk <= E");
  if (E > wdb::ROUTER_PER * 32 || topk > wdb::ROUTER_MAX_K)
    return fail(WD_ERR_UNSUPPORTED, "router supports E <= 1024 and topk <= 32");
  if (B == 0) return WD_OK;
  if (!logits || !topk_ids || !topk_weights) return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(logits) & (logits_fp32 ? 3u : 1u)) != 0 ||
      (reinterpret_cast<uintptr_t>(topk_ids) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(topk_weights) & 3u) != 0)
    return fail(WD_ERR_ALIGNMENT, "logits / topk_ids / topk_weights misaligned for their type");
  wdb::RouterArgs a;
  a.logits = logits;
  a.logits_fp32 = logits_fp32 ? 1 : 0;
  a.ids = topk_ids;
  a.weights = topk_weights;
  a.B = B; a.E = E; a.K = topk;
  a.renormalize = renormalize ? 1 : 0;
  const unsigned grid = (unsigned)((B + wdb::ROUTER_WARPS - 1) / wdb::ROUTER_WARPS);
  wdb::moe_router_topk_kernel<<<grid, wdb::ROUTER_WARPS * 32, 0,
                                reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return fail(WD_ERR_CUDA, std::string("router launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

int wd_copy_ranges(const void* const* src, void* const* dst, const size_t* bytes, int n,
                   void* stream) {
  g_last_error.clear();
  if (n < 0 || n > wdb::COPY_MAX_RANGES) return fail(WD_ERR_SHAPE, "need 0 <= n <= 4 ranges");
  if (n > 0 && (!src || !dst || !bytes)) return fail(WD_ERR_NULL_POINTER, "null range array");
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(WD_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  wdb::CopyRanges c{};
  c.first[0] = 0;
  int m = 0;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    if (!src[i] || !dst[i]) return fail(WD_ERR_NULL_POINTER, "null range pointer");
    unsigned char *s = nullptr, *d = nullptr;
    int rc = device_view(src[i], dev, "src", &s);
    if (rc != WD_OK) return rc;
    rc = device_view(dst[i], dev, "dst", &d);
    if (rc != WD_OK) return rc;
    c.src[m] = s;
    c.dst[m] = d;
    c.bytes[m] = bytes[i];
    c.vec[m] = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0;
    c.first[m + 1] = c.first[m] + (bytes[i] + 15) / 16;
    ++m;
  }
  c.n = m;
  if (m == 0) return WD_OK;
  DeviceInfo* di = nullptr;
  const int rc = device_info(&di);
  if (rc != WD_OK) return rc;
  const unsigned long long units = c.first[m];
  const unsigned long long per_cta = (unsigned long long)wdb::COPY_THREADS * wdb::COPY_UNROLL;
  const unsigned grid = (unsigned)std::min<unsigned long long>((units + per_cta - 1) / per_cta,
                                                               (unsigned long long)di->sm_count * 4);
  wdb::copy_ranges_kernel<<<grid, wdb::COPY_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(c);
  err = cudaGetLastError();
  if (err != cudaSuccess) return fail(WD_ERR_CUDA, std::string("copy launch: ") + cudaGetErrorString(err));
  note_launch();
  return WD_OK;
}

int wd_set_ffn_path(int path) {
  g_last_error.clear();
  if (path < 0 || path > 3)
    return fail(WD_ERR_SHAPE, "path must be 0 (auto), 1 (split), 2 (fused) or 3 (tensor-core fused)");
  g_ffn_path.store(path);
  return WD_OK;
}

int wd_moe_ffn_3d_batched_kernels(int B, int E, int topk, int hidden, int inter, int* kind) {
  g_last_error.clear();
  if (!kind) return fail(WD_ERR_NULL_POINTER, "kind is NULL");
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  *kind = WD_FFN_KERNELS_SPLIT;
  if (B == 0) return WD_OK;
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  const int fp = ffn_path();
  FfnPlan plan;
  FfnTcPlan tplan;
  if ((fp == 0 || fp == 2) &&
      ffn_plan(dev, B, E, topk, hidden, inter,
               fp == 2 ? wdb::FFN_MAX_SLOTS : WD_FFN_AUTO_MAX_SLOTS, &plan))
    *kind = WD_FFN_KERNELS_SIMT_SINGLE;
  else if ((fp == 3 || fp == 0) && !dev->ffn_tc_off &&
           ffn_tc_plan(dev, B, E, topk, hidden, inter, &tplan) &&
           (fp == 3 || ffn_tc_auto(tplan, B, topk, inter)))
    *kind = WD_FFN_KERNELS_TC_SINGLE;
  return WD_OK;
}

int wd_moe_ffn_3d_batched(const void* x, const void* w_gate_up, const void* w_down,
                          const int32_t* topk_ids, const float* topk_scale, void* h_buf,
                          uint32_t* sync, void* y_out, int out_fp32, int B, int E, int topk,
                          int hidden, int inter, uint32_t* status, void* stream) {
  g_last_error.clear();
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (hidden % 8 != 0 || inter % 8 != 0)
    return fail(WD_ERR_SHAPE, "hidden and inter must be multiples of 8 (16-byte weight rows)");
  if (B == 0) return WD_OK;
  if (!x || !w_gate_up || !w_down || !topk_ids || !topk_scale || !h_buf || !y_out)
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down) || !aligned16(h_buf))
    return fail(WD_ERR_ALIGNMENT, "x, w_gate_up, w_down and h_buf must be 16-byte aligned");
  if (sync && (reinterpret_cast<uintptr_t>(sync) & 7u) != 0)
    return fail(WD_ERR_ALIGNMENT, "sync must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  FfnPlan plan;
  const int fp = ffn_path();
  uint32_t* const bar = sync ? sync : reinterpret_cast<uint32_t*>(dev->ffn_sync);
  if ((fp == 0 || fp == 2) &&
      ffn_plan(dev, B, E, topk, hidden, inter,
               fp == 2 ? wdb::FFN_MAX_SLOTS : WD_FFN_AUTO_MAX_SLOTS, &plan))
    return ffn_launch(dev, plan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf, bar, y_out,
                      out_fp32, B, E, topk, hidden, inter,
                      status, reinterpret_cast<cudaStream_t>(stream));
  FfnTcPlan tplan;
  if ((fp == 3 || fp == 0) && !dev->ffn_tc_off &&
      ffn_tc_plan(dev, B, E, topk, hidden, inter, &tplan) &&
      (fp == 3 || ffn_tc_auto(tplan, B, topk, inter))) {
    rc = ffn_tc_launch(dev, tplan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf,
                       reinterpret_cast<unsigned long long*>(bar), y_out, out_fp32, B, E, topk,
                       hidden, inter, status, reinterpret_cast<cudaStream_t>(stream));
    if (rc != WD_ERR_UNSUPPORTED) return rc;
    dev->ffn_tc_off = true;  // the runtime refused the cooperative cluster launch: not again
    g_last_error.clear();
  }
  rc = gate_up_impl<wdb::W_BF16>(x, reinterpret_cast<const uint8_t*>(w_gate_up), nullptr,
                                 topk_ids, h_buf, B, E, topk, hidden, inter, status, stream);
  if (rc) return rc;
  return down_impl<wdb::W_BF16>(h_buf, reinterpret_cast<const uint8_t*>(w_down), nullptr,
                                topk_ids, topk_scale, y_out, out_fp32, B, E, topk, hidden, inter,
                                status, stream);
}

int wd_moe_ffn_3d_batched_noalloc(const void* x, const void* w_gate_up, const void* w_down,
                                  const int32_t* topk_ids, const float* topk_scale, void* y_out,
                                  int out_fp32, int B, int E, int topk, int hidden, int inter,
                                  uint32_t* status, void* stream) {
  g_last_error.clear();
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (hidden % 8 != 0 || inter % 8 != 0)
    return fail(WD_ERR_SHAPE, "hidden and inter must be multiples of 8 (16-byte weight rows)");
  if (B == 0) return WD_OK;
  if ((size_t)B * topk * inter * 2 > kNoallocHBytes)
    return fail(WD_ERR_UNSUPPORTED, "B*topk*inter*2 exceeds the 131072-byte static scratch");
  if (!x || !w_gate_up || !w_down || !topk_ids || !topk_scale || !y_out)
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down))
    return fail(WD_ERR_ALIGNMENT, "x, w_gate_up and w_down must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!dev->noalloc_scratch) {
      const cudaError_t err =
          cudaGetSymbolAddress(reinterpret_cast<void**>(&dev->noalloc_scratch), g_wd_noalloc_scratch);
      if (err != cudaSuccess)
        return fail(WD_ERR_CUDA, std::string("scratch address: ") + cudaGetErrorString(err));
    }
  }
  uint32_t* sync = reinterpret_cast<uint32_t*>(dev->noalloc_scratch);
  void* h_buf = dev->noalloc_scratch + kNoallocHeader;
  FfnPlan plan;
  const int fp = ffn_path();
  if ((fp == 0 || fp == 2) &&
      ffn_plan(dev, B, E, topk, hidden, inter,
               fp == 2 ? wdb::FFN_MAX_SLOTS : WD_FFN_AUTO_MAX_SLOTS, &plan))
    return ffn_launch(dev, plan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf, sync, y_out,
                      out_fp32, B, E, topk, hidden, inter, status,
                      reinterpret_cast<cudaStream_t>(stream));
  FfnTcPlan tplan;
  if ((fp == 3 || fp == 0) && !dev->ffn_tc_off &&
      ffn_tc_plan(dev, B, E, topk, hidden, inter, &tplan) &&
      (fp == 3 || ffn_tc_auto(tplan, B, topk, inter))) {
    rc = ffn_tc_launch(dev, tplan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf,
                       reinterpret_cast<unsigned long long*>(sync), y_out, out_fp32, B, E, topk,
                       hidden, inter, status, reinterpret_cast<cudaStream_t>(stream));
    if (rc != WD_ERR_UNSUPPORTED) return rc;
    dev->ffn_tc_off = true;
    g_last_error.clear();
  }
  rc = gate_up_impl<wdb::W_BF16>(x, reinterpret_cast<const uint8_t*>(w_gate_up), nullptr,
                                 topk_ids, h_buf, B, E, topk, hidden, inter, status, stream);
  if (rc) return rc;
  return down_impl<wdb::W_BF16>(h_buf, reinterpret_cast<const uint8_t*>(w_down), nullptr,
                                topk_ids, topk_scale, y_out, out_fp32, B, E, topk, hidden, inter,
                                status, stream);
}

int wd_tp_comm_create(int world, int rank, int max_tokens, int hidden, void** comm,
                      void* ipc_handle) {
  g_last_error.clear();
  if (!comm || !ipc_handle) return fail(WD_ERR_NULL_POINTER, "comm and ipc_handle are required");
  *comm = nullptr;
  if (world < 2 || world > wdb::TP_MAX_WORLD || rank < 0 || rank >= world)
    return fail(WD_ERR_SHAPE, "world must be 2..8 and 0 <= rank < world");
  if (max_tokens < 1 || hidden < 4 || hidden % 4 != 0)
    return fail(WD_ERR_SHAPE, "max_tokens >= 1 and hidden % 4 == 0 required");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  TpComm* c = new TpComm();
  cudaGetDevice(&c->device);
  c->world = world; c->rank = rank; c->max_tokens = max_tokens; c->hidden = hidden;
  c->max_ctas = dev->sm_count;
  c->recv_bytes = ((size_t)2 * world * max_tokens * hidden * 8 + 255) / 256 * 256;
  cudaError_t err = cudaMalloc(&c->block, c->recv_bytes);
  if (err == cudaSuccess) err = cudaMemset(c->block, 0, c->recv_bytes);
  if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(&c->epochs), c->max_ctas * 4);
  if (err == cudaSuccess) err = cudaMemset(c->epochs, 0, c->max_ctas * 4);
  if (err == cudaSuccess)
    err = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), c->block);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    if (c->block) cudaFree(c->block);
    if (c->epochs) cudaFree(c->epochs);
    delete c;
    return fail(WD_ERR_CUDA, std::string("tp comm create: ") + cudaGetErrorString(err));
  }
  *comm = c;
  return WD_OK;
}

int wd_tp_comm_open(void* comm, const void* ipc_handles) {
  g_last_error.clear();
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c || !ipc_handles) return fail(WD_ERR_NULL_POINTER, "comm and ipc_handles are required");
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(ipc_handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->peer[r]) continue;
    const cudaError_t err =
        cudaIpcOpenMemHandle(&c->peer[r], hs[r], cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess)
      return fail(WD_ERR_CUDA, std::string("tp comm open (rank ") + std::to_string(r) +
                                   "): " + cudaGetErrorString(err));
  }
  return WD_OK;
}

int wd_tp_comm_set_exchange(void* comm, int mode) {
  g_last_error.clear();
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c) return fail(WD_ERR_NULL_POINTER, "comm is NULL");
  if (mode < 0 || mode > 2)
    return fail(WD_ERR_SHAPE, "mode must be 0 (by size), 1 (one-shot) or 2 (two-shot)");
  c->exchange = mode;
  return WD_OK;
}

int wd_tp_comm_destroy(void* comm) {
  g_last_error.clear();
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c) return WD_OK;
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
  cudaFree(c->block);
  cudaFree(c->epochs);
  delete c;
  return WD_OK;
}

int wd_moe_down_3d_batched_allreduce(const void* h, const void* w_down, const int32_t* topk_ids,
                                     const float* topk_scale, void* y_out, int B, int E, int topk,
                                     int hidden, int inter, void* comm, uint32_t* status,
                                     void* stream) {
  g_last_error.clear();
  TpComm* c = static_cast<TpComm*>(comm);
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (!c) return fail(WD_ERR_NULL_POINTER, "comm is NULL");
  if (B == 0) return WD_OK;
  if (!h || !w_down || !topk_ids || !topk_scale || !y_out)
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(h) || !aligned16(w_down) || inter % 8 != 0)
    return fail(WD_ERR_ALIGNMENT, "h and w_down must be 16-byte aligned, inter % 8 == 0");
  if (hidden != c->hidden) return fail(WD_ERR_SHAPE, "hidden differs from the communicator's");
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && !c->peer[r]) return fail(WD_ERR_UNSUPPORTED, "communicator not opened");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  if (E > wdb::MAX_DEDUP_E || inter > wdb::DTC_MAXKC * wdb::DTC_BK ||
      (hidden + wdb::DTC_M - 1) / wdb::DTC_M > dev->sm_count)
    return fail(WD_ERR_UNSUPPORTED, "shape outside the tensor-core down kernel (inter <= 2048)");
  const int tb = std::min(std::max(1, wdb::MAX_SLOTS / topk), std::min(64, c->max_tokens));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tb) {
    const int bn = std::min(tb, B - b0);
    const wdb::TpArgs tp = make_tp_args(c, bn);
    rc = down_tc_launch(dev, reinterpret_cast<const __nv_bfloat16*>(h) + (size_t)b0 * topk * inter,
                        w_down, topk_ids + (size_t)b0 * topk, topk_scale + (size_t)b0 * topk,
                        reinterpret_cast<__nv_bfloat16*>(y_out) + (size_t)b0 * hidden, 0, bn, E,
                        topk, hidden, inter, status, s, &tp);
    if (rc) return rc;
  }
  return WD_OK;
}

int wd_moe_ffn_3d_batched_allreduce(const void* x, const void* w_gate_up, const void* w_down,
                                    const int32_t* topk_ids, const float* topk_scale, void* h_buf,
                                    uint32_t* sync, void* y_out, int B, int E, int topk,
                                    int hidden, int inter, void* comm, uint32_t* status,
                                    void* stream) {
  g_last_error.clear();
  TpComm* c = static_cast<TpComm*>(comm);
  int rc = check_common(B, E, topk, hidden, inter);
  if (rc) return rc;
  if (!c) return fail(WD_ERR_NULL_POINTER, "comm is NULL");
  if (hidden % 8 != 0 || inter % 8 != 0)
    return fail(WD_ERR_SHAPE, "hidden and inter must be multiples of 8 (16-byte weight rows)");
  if (B == 0) return WD_OK;
  if (!x || !w_gate_up || !w_down || !topk_ids || !topk_scale || !h_buf || !y_out)
    return fail(WD_ERR_NULL_POINTER, "null tensor pointer");
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down) || !aligned16(h_buf))
    return fail(WD_ERR_ALIGNMENT, "x, w_gate_up, w_down and h_buf must be 16-byte aligned");
  if (sync && (reinterpret_cast<uintptr_t>(sync) & 7u) != 0)
    return fail(WD_ERR_ALIGNMENT, "sync must be 8-byte aligned");
  if (hidden != c->hidden) return fail(WD_ERR_SHAPE, "hidden differs from the communicator's");
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && !c->peer[r]) return fail(WD_ERR_UNSUPPORTED, "communicator not opened");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  FfnPlan plan;
  const int fp = ffn_path();
  if ((fp == 0 || fp == 2) && B <= c->max_tokens &&
      ffn_plan(dev, B, E, topk, hidden, inter,
               fp == 2 ? wdb::FFN_MAX_SLOTS : WD_FFN_AUTO_MAX_SLOTS, &plan) &&
      plan.grid <= c->max_ctas) {
    const wdb::TpArgs tp = make_tp_args(c, B);
    return ffn_launch(dev, plan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf,
                      sync ? sync : reinterpret_cast<uint32_t*>(dev->ffn_sync), y_out, 0, B, E,
                      topk, hidden, inter, status, reinterpret_cast<cudaStream_t>(stream), &tp);
  }
  FfnTcPlan tplan;
  if (B <= c->max_tokens && (fp == 3 || fp == 0) && !dev->ffn_tc_off &&
      ffn_tc_plan(dev, B, E, topk, hidden, inter, &tplan) &&
      (fp == 3 || ffn_tc_auto(tplan, B, topk, inter)) && tplan.tiles * tplan.cl <= c->max_ctas) {
    const wdb::TpArgs tp = make_tp_args(c, B);
    rc = ffn_tc_launch(dev, tplan, x, w_gate_up, w_down, topk_ids, topk_scale, h_buf,
                       reinterpret_cast<unsigned long long*>(
                           sync ? sync : reinterpret_cast<uint32_t*>(dev->ffn_sync)),
                       y_out, 0, B, E, topk, hidden, inter, status,
                       reinterpret_cast<cudaStream_t>(stream), &tp);
    if (rc != WD_ERR_UNSUPPORTED) return rc;
    dev->ffn_tc_off = true;
    g_last_error.clear();
  }
  rc = gate_up_impl<wdb::W_BF16>(x, reinterpret_cast<const uint8_t*>(w_gate_up), nullptr,
                                 topk_ids, h_buf, B, E, topk, hidden, inter, status, stream);
  if (rc) return rc;
  return wd_moe_down_3d_batched_allreduce(h_buf, w_down, topk_ids, topk_scale, y_out, B, E, topk,
                                          hidden, inter, comm, status, stream);
}

int wd_status_read(uint32_t* value, int clear) {
  g_last_error.clear();
  if (!value) return fail(WD_ERR_NULL_POINTER, "value is NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(value, wdb::g_wd_status, sizeof(uint32_t));
  if (err == cudaSuccess && clear) {
    const uint32_t zero = 0u;
    err = cudaMemcpyToSymbol(wdb::g_wd_status, &zero, sizeof(uint32_t));
  }
  if (err != cudaSuccess) return fail(WD_ERR_CUDA, std::string("status read: ") + cudaGetErrorString(err));
  return WD_OK;
}

}  // extern "C"
