// Small host <-> device transfers done by the GPU's own loads and stores.
//
// A decode step moves a few KB to a few hundred KB each way (x, topk_ids and
// topk_scale in, y out).  At those sizes a copy-engine transfer from
// page-locked host memory is dominated by its fixed start-up cost; one
// kernel whose threads each load and store 16-byte units over PCIe (host
// memory through its device mapping) has many reads in flight at once and no
// copy-engine hand-off.  No counterpart in the reference, whose API takes
// device tensors only.
#pragma once

#include <cstdint>

namespace wdb {

constexpr int COPY_MAX_RANGES = 4;
constexpr int COPY_THREADS = 256;
constexpr int COPY_UNROLL = 4;  // 16-byte units per thread per round (loads before stores)

// Up to COPY_MAX_RANGES byte ranges, src[i] -> dst[i] (device-visible
// addresses).  first[i] = 16-byte units before range i; vec[i] = both
// pointers 16-byte aligned (else the range is copied byte by byte).
struct CopyRanges {
  const unsigned char* src[COPY_MAX_RANGES];
  unsigned char* dst[COPY_MAX_RANGES];
  unsigned long long bytes[COPY_MAX_RANGES];
  unsigned long long first[COPY_MAX_RANGES + 1];
  int vec[COPY_MAX_RANGES];
  int n;
};

__global__ void __launch_bounds__(COPY_THREADS) copy_ranges_kernel(const CopyRanges c) {
  const unsigned long long total = c.first[c.n];
  const unsigned long long stride = (unsigned long long)gridDim.x * COPY_THREADS;
  for (unsigned long long u0 = (unsigned long long)blockIdx.x * COPY_THREADS + threadIdx.x;
       u0 < total; u0 += COPY_UNROLL * stride) {
    uint4 v[COPY_UNROLL];
    int rg[COPY_UNROLL];
    unsigned long long off[COPY_UNROLL];
    bool whole[COPY_UNROLL];
#pragma unroll
    for (int k = 0; k < COPY_UNROLL; ++k) {
      const unsigned long long u = u0 + k * stride;
      rg[k] = -1;
      whole[k] = false;
      if (u < total) {
        int g = 0;
        while (g + 1 < c.n && u >= c.first[g + 1]) ++g;
        rg[k] = g;
        off[k] = (u - c.first[g]) * 16ull;
        whole[k] = c.vec[g] && off[k] + 16ull <= c.bytes[g];
        if (whole[k]) v[k] = *reinterpret_cast<const uint4*>(c.src[g] + off[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < COPY_UNROLL; ++k) {
      if (rg[k] < 0) continue;
      const int g = rg[k];
      if (whole[k]) {
        *reinterpret_cast<uint4*>(c.dst[g] + off[k]) = v[k];
      } else {
        const unsigned long long end = min(off[k] + 16ull, c.bytes[g]);
        for (unsigned long long b = off[k]; b < end; ++b) c.dst[g][b] = c.src[g][b];
      }
    }
  }
}

}  // namespace wdb
