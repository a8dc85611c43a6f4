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
// One thread per 2x2 patch writes its 12 outputs (12 coalesced planes); a CTA
// of 32 x 8 patches builds its tile's axis plans once in shared memory. Every
// value is computed in the CPU path's exact operation order with explicitly
// rounded IEEE operations (no FMA contraction), so the output equals
// compose_and_patchify bit for bit:
//   axis plan (vae.cpp:26-42): scale = r / s, filter = max(1, 1 / scale),
//     centre = (p + 0.5) / scale - 0.5, taps ceil(c - f) .. floor(c + f),
//     weight max(0, 1 - |i - c| / f), zero weights dropped, then w / sum;
//   horizontal pass over the source row, then vertical pass (vae.cpp:59-87),
//   each a running sum of value * weight from 0; U8 reads value * (1 / 255).
#include <algorithm>
#include <cmath>
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

// Canvas pixel (cx, cy) from its view directly: the axis plans are rebuilt per
// pixel. Used for tiles that straddle two views and for very large downscales.
__device__ __forceinline__ void pixel_direct(const ViewsDev& views, int cx, int cy, int out_w,
                                             int out_h, float (&acc)[3]) {
  const Cell cell = cell_of(cx, cy, out_w, out_h);
  const ViewDev v = views.v[cell.view];
  // resize_center_crop's plan key (vae.cpp:14-22).
  const float scale = fmaxf(__fdiv_rn(static_cast<float>(cell.w), static_cast<float>(v.w)),
                            __fdiv_rn(static_cast<float>(cell.h), static_cast<float>(v.h)));
  const int rw = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.w), scale)));
  const int rh = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.h), scale)));
  const Axis ax = make_axis(cell.x + (rw - cell.w) / 2, v.w, rw);
  const Axis ay = make_axis(cell.y + (rh - cell.h) / 2, v.h, rh);
  acc[0] = acc[1] = acc[2] = 0.0f;
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
}

// Axis plan of one output position into shared memory: the clamped source
// index and normalised weight of every non-zero tap, in tap order (what
// resize_center_crop stores per position, vae.cpp:31-40). Returns the count.
__device__ __forceinline__ int plan_axis(int p, int source, int resized, int* idx, float* w,
                                         int kmax) {
  const Axis a = make_axis(p, source, resized);
  int n = 0;
  for (int i = a.first; i <= a.last && n < kmax; ++i) {
    const float t = tap_weight(i, a.center, a.filter);
    if (t == 0.0f) continue;
    idx[n] = max(0, min(source - 1, i));
    w[n] = __fdiv_rn(t, a.total);
    ++n;
  }
  return n;
}

constexpr int kTPW = 32, kTPH = 8;  // patches per CTA: 64 x 16 canvas pixels
constexpr int kPlans = 2 * kTPW + 2 * kTPH;

// One CTA = 32 x 8 patches. When the tile lies in one view (every tile of a
// canvas whose half sizes are multiples of 64 x 16, e.g. config 2), the
// tile's 64 column plans and 16 row plans are built once in shared memory
// and every pixel reuses them; otherwise each pixel builds its own.
__global__ void __launch_bounds__(256) preprocess_kernel(ViewsDev views, int out_w, int out_h,
                                                         float* __restrict__ out, int kmax) {
  extern __shared__ uint8_t smem[];
  int* s_idx = reinterpret_cast<int*>(smem);
  float* s_w = reinterpret_cast<float*>(s_idx + kPlans * kmax);
  int* s_n = reinterpret_cast<int*>(s_w + kPlans * kmax);
  const int pw = out_w / 2, ph = out_h / 2;
  const int tx = threadIdx.x % kTPW, ty = threadIdx.x / kTPW;
  const int px = blockIdx.x * kTPW + tx, py = blockIdx.y * kTPH + ty;
  const int cx0 = 2 * blockIdx.x * kTPW, cy0 = 2 * blockIdx.y * kTPH;
  const int cx1 = min(out_w, cx0 + 2 * kTPW) - 1, cy1 = min(out_h, cy0 + 2 * kTPH) - 1;
  const Cell c00 = cell_of(cx0, cy0, out_w, out_h);
  const bool uniform = kmax > 0 && c00.view == cell_of(cx1, cy0, out_w, out_h).view &&
                       c00.view == cell_of(cx0, cy1, out_w, out_h).view &&
                       c00.view == cell_of(cx1, cy1, out_w, out_h).view;
  const size_t plane = static_cast<size_t>(pw) * ph;
  const size_t o = static_cast<size_t>(py) * pw + px;
  if (!uniform) {
    if (px >= pw || py >= ph) return;
#pragma unroll
    for (int dx = 0; dx < 2; ++dx)
#pragma unroll
      for (int dy = 0; dy < 2; ++dy) {
        float acc[3];
        pixel_direct(views, 2 * px + dx, 2 * py + dy, out_w, out_h, acc);
#pragma unroll
        for (int c = 0; c < 3; ++c)
          out[static_cast<size_t>((c * 2 + dx) * 2 + dy) * plane + o] =
              __fsub_rn(__fmul_rn(acc[c], 2.0f), 1.0f);
      }
    return;
  }
  const ViewDev v = views.v[c00.view];
  const float scale = fmaxf(__fdiv_rn(static_cast<float>(c00.w), static_cast<float>(v.w)),
                            __fdiv_rn(static_cast<float>(c00.h), static_cast<float>(v.h)));
  const int rw = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.w), scale)));
  const int rh = static_cast<int>(roundf(__fmul_rn(static_cast<float>(v.h), scale)));
  const int t = threadIdx.x;
  if (t < 2 * kTPW) {
    if (cx0 + t < out_w)
      s_n[t] = plan_axis(c00.x + t + (rw - c00.w) / 2, v.w, rw, s_idx + t * kmax, s_w + t * kmax, kmax);
  } else if (t < kPlans) {
    const int r = t - 2 * kTPW;
    if (cy0 + r < out_h)
      s_n[t] = plan_axis(c00.y + r + (rh - c00.h) / 2, v.h, rh, s_idx + t * kmax, s_w + t * kmax,
                         kmax);
  }
  __syncthreads();
  if (px >= pw || py >= ph) return;
#pragma unroll
  for (int dx = 0; dx < 2; ++dx) {
    const int xs = 2 * tx + dx;
    const int nx = s_n[xs];
    const int* xi = s_idx + xs * kmax;
    const float* xw = s_w + xs * kmax;
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
      const int ys = 2 * kTPW + 2 * ty + dy;
      const int ny = s_n[ys];
      float acc[3] = {0.0f, 0.0f, 0.0f};
      for (int j = 0; j < ny; ++j) {
        const int yy = s_idx[ys * kmax + j];
        float hor[3] = {0.0f, 0.0f, 0.0f};
        for (int i = 0; i < nx; ++i) {
          float rgb[3];
          read_rgb(v, xi[i], yy, rgb);
          const float wn = xw[i];
#pragma unroll
          for (int c = 0; c < 3; ++c) hor[c] = __fadd_rn(hor[c], __fmul_rn(rgb[c], wn));
        }
        const float wyn = s_w[ys * kmax + j];
#pragma unroll
        for (int c = 0; c < 3; ++c) acc[c] = __fadd_rn(acc[c], __fmul_rn(hor[c], wyn));
      }
#pragma unroll
      for (int c = 0; c < 3; ++c)
        out[static_cast<size_t>((c * 2 + dx) * 2 + dy) * plane + o] =
            __fsub_rn(__fmul_rn(acc[c], 2.0f), 1.0f);
    }
  }
}

}  // namespace

bool launch_preprocess(const PreprocessView* views, int out_w, int out_h, float* out,
                       cudaStream_t stream) {
  ViewsDev d;
  for (int i = 0; i < 3; ++i) d.v[i] = ViewDev{views[i].data, views[i].w, views[i].h, views[i].format};
  // Taps per plan: at most 2 * filter + 1 with filter = max(1, source / resized)
  // (build_axis, vae.cpp:26-42); a margin covers the float rounding of the scale.
  const int top = out_h / 2, left = out_w / 2;
  const int cw[3] = {out_w, left, out_w - left}, ch[3] = {top, out_h - top, out_h - top};
  double fmax = 1.0;
  for (int i = 0; i < 3; ++i) {
    const float scale = std::max(static_cast<float>(cw[i]) / views[i].w,
                                 static_cast<float>(ch[i]) / views[i].h);
    const double rw = std::max(1.0, std::round(static_cast<double>(views[i].w) * scale));
    const double rh = std::max(1.0, std::round(static_cast<double>(views[i].h) * scale));
    fmax = std::max(fmax, std::max(views[i].w / rw, views[i].h / rh));
  }
  int kmax = static_cast<int>(2.0 * fmax) + 4;
  // Shared plans up to 48 KB (kmax <= 72); beyond, every pixel builds its own.
  if (static_cast<size_t>(kPlans) * kmax * 8 + kPlans * 4 > 48 * 1024) kmax = 0;
  const size_t smem = kmax > 0 ? static_cast<size_t>(kPlans) * kmax * 8 + kPlans * 4 : 0;
  const int pw = out_w / 2, ph = out_h / 2;
  const dim3 grid((pw + kTPW - 1) / kTPW, (ph + kTPH - 1) / kTPH);
  preprocess_kernel<<<grid, kTPW * kTPH, smem, stream>>>(d, out_w, out_h, out, kmax);
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace wamb
