// L2 prefetch of upcoming weight ranges, shared by the non-GEMM kernels.
#pragma once

#include "kernels.h"
#include "ptx.cuh"

namespace wamb {

// CTA `cta` of `ncta` prefetches its share of the ranges into L2 (called by one
// thread per CTA, before griddepcontrol.wait: weights never depend on the
// preceding kernel).
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int cta, int ncta) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!pf.ptr[r] || pf.bytes[r] <= 0) continue;
    const long long per = ((pf.bytes[r] + ncta - 1) / ncta + 15) & ~15ll;
    const long long start = per * cta;
    long long left = pf.bytes[r] - start;
    if (left > per) left = per;
    const char* p = static_cast<const char*>(pf.ptr[r]) + start;
    while (left > 0) {
      const uint32_t n = static_cast<uint32_t>(left > 65536 ? 65536 : left);
      prefetch_l2_bulk(p, n);
      p += n;
      left -= n;
    }
  }
}

}  // namespace wamb
