// Vision front-end, stage 1: compose the three camera views onto one canvas
// (resize to cover + centre crop, triangle filter), patchify 2x2 and map to
// [-1, 1]. Replaces the reference's compose_and_patchify / resize_center_crop
// (src/models/gwp05/engine/vae.cpp:1-134) and its CUDA twin preprocess_kernel
// (src/models/gwp05/kernels/cuda_preprocess.cu:45-137).
//
// Canvas layout (vae.cpp:104-110): view 0 fills the top half (width W, height
// H/2); views 1 and 2 split the bottom half left / right. Output [12][H/2][W/2]
// F32, packed channel (c * 2 + dx) * 2 + dy for canvas pixel (2x + dx, 2y + dy).
//
// One thread per 2x2 patch writes its 12 outputs (12 coalesced planes). Every
// value is computed in the CPU path's exact operation order with explicitly
// rounded IEEE operations (no FMA contraction), so the output equals
// compose_and_patchify bit for bit:
//   axis plan (vae.cpp:26-42): scale = r / s, filter = max(1, 1 / scale),
//     centre = (p + 0.5) / scale - 0.5, taps ceil(c - f) .. floor(c + f),
//     weight max(0, 1 - |i - c| / f), zero weights dropped, then w / sum;
//   horizontal pass over the source row, then vertical pass (vae.cpp:59-87),
//   each a running sum of value * weight from 0; U8 reads value * (1 / 255).
#include <cstdint>

#include "kernels.h"

namespace wamb {
namespace {

struct ViewDev {
  const void* data;
  int w, h, format;  // format 0: U8 RGB, 1: F32 RGB in [0, 1]
};

struct ViewsDev {
  ViewDev v[3];
};

struct Axis {
  int first, last;
  float center, filter, total;
};

__device__ __forceinline__ float tap_weight(int i, float center, float filter) {
  return fmaxf(0.0f, __fsub_rn(1.0f, __fdiv_rn(fabsf(__fsub_rn(static_cast<float>(i), center)),
                                               filter)));
}

// build_axis (vae.cpp:26-42) for output position p (crop offset included).
__device__ __forceinline__ Axis make_axis(int p, int source, int resized) {
  Axis a;
  const float scale = __fdiv_rn(static_cast<float>(resized), static_cast<float>(source));
  a.filter = fmaxf(1.0f, __fdiv_rn(1.0f, scale));
  a.center = __fsub_rn(__fdiv_rn(__fadd_rn(static_cast<float>(p), 0.5f), scale), 0.5f);
  a.first = static_cast<int>(ceilf(__fsub_rn(a.center, a.filter)));
  a.last = static_cast<int>(floorf(__fadd_rn(a.center, a.filter)));
  float total = 0.0f;
  for (int i = a.first; i <= a.last; ++i) {
    const float w = tap_weight(i, a.center, a.filter);
    if (w != 0.0f) total = __fadd_rn(total, w);
  }
  a.total = total;
  return a;
}

__device__ __forceinline__ void read_rgb(const ViewDev& v, int x, int y, float (&rgb)[3]) {
  const size_t idx = (static_cast<size_t>(y) * v.w + x) * 3;
  if (v.format == 0) {
    const uint8_t* p = static_cast<const uint8_t*>(v.data) + idx;
#pragma unroll
    for (int c = 0; c < 3; ++c) rgb[c] = __fmul_rn(static_cast<float>(p[c]), 1.0f / 255.0f);
  } else {
    const float* p = static_cast<const float*>(v.data) + idx;
#pragma unroll
    for (int c = 0; c < 3; ++c) rgb[c] = p[c];
  }
}

// View, cell size and position inside the cell of canvas pixel (cx, cy)
// (vae.cpp:104-110 / cuda_preprocess.cu:72-106).
struct Cell {
  int view, w, h, x, y;
};

__device__ __forceinline__ Cell cell_of(int cx, int cy, int out_w, int out_h) {
  const int top_h = out_h / 2, left_w = out_w / 2;
  if (cy < top_h) return Cell{0, out_w, top_h, cx, cy};
  if (cx < left_w) return Cell{1, left_w, out_h - top_h, cx, cy - top_h};
  return Cell{2, out_w - left_w, out_h - top_h, cx - left_w, cy - top_h};
}

__global__ void __launch_bounds__(128) preprocess_kernel(ViewsDev views, int out_w, int out_h,
                                                         float* __restrict__ out) {
  const int pw = out_w / 2, ph = out_h / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= pw * ph) return;
  const int px = idx % pw, py = idx / pw;
  const size_t plane = static_cast<size_t>(pw) * ph;
#pragma unroll
  for (int dx = 0; dx < 2; ++dx) {
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
      // Each canvas pixel on its own: with H/2 or W/2 odd a patch can span two views.
      const Cell cell = cell_of(2 * px + dx, 2 * py + dy, out_w, out_h);
      const ViewDev v = views.v[cell.view];
      // resize_center_crop's plan key (vae.cpp:14-22).
      const float scale = fmaxf(__fdiv_rn(static_cast<float>(cell.w), static_cast<float>(v.w)),
                                __fdiv_rn(static_cast<float>(cell.h), static_cast<float>(v.h)));
      const int rw = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.w), scale)));
      const int rh = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.h), scale)));
      const Axis ax = make_axis(cell.x + (rw - cell.w) / 2, v.w, rw);
      const Axis ay = make_axis(cell.y + (rh - cell.h) / 2, v.h, rh);
      float acc[3] = {0.0f, 0.0f, 0.0f};
      for (int sy = ay.first; sy <= ay.last; ++sy) {
        const float wy = tap_weight(sy, ay.center, ay.filter);
        if (wy == 0.0f) continue;
        const int yy = max(0, min(v.h - 1, sy));
        float hor[3] = {0.0f, 0.0f, 0.0f};
        for (int sx = ax.first; sx <= ax.last; ++sx) {
          const float wx = tap_weight(sx, ax.center, ax.filter);
          if (wx == 0.0f) continue;
          const float wn = __fdiv_rn(wx, ax.total);
          float rgb[3];
          read_rgb(v, max(0, min(v.w - 1, sx)), yy, rgb);
#pragma unroll
          for (int c = 0; c < 3; ++c) hor[c] = __fadd_rn(hor[c], __fmul_rn(rgb[c], wn));
        }
        const float wyn = __fdiv_rn(wy, ay.total);
#pragma unroll
        for (int c = 0; c < 3; ++c) acc[c] = __fadd_rn(acc[c], __fmul_rn(hor[c], wyn));
      }
#pragma unroll
      for (int c = 0; c < 3; ++c)
        out[static_cast<size_t>((c * 2 + dx) * 2 + dy) * plane + idx] =
            __fsub_rn(__fmul_rn(acc[c], 2.0f), 1.0f);
    }
  }
}

}  // namespace

bool launch_preprocess(const PreprocessView* views, int out_w, int out_h, float* out,
                       cudaStream_t stream) {
  ViewsDev d;
  for (int i = 0; i < 3; ++i) d.v[i] = ViewDev{views[i].data, views[i].w, views[i].h, views[i].format};
  const int patches = (out_w / 2) * (out_h / 2);
  preprocess_kernel<<<(patches + 127) / 128, 128, 0, stream>>>(d, out_w, out_h, out);
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace wamb
