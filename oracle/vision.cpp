// CPU oracle (TEST INFRASTRUCTURE ONLY) of the vision front-end's first stage:
// three views composed onto the canvas, each resized to cover its cell with a
// triangle (bilinear-antialias) filter and centre cropped, then patchified 2x2
// and mapped to [-1, 1]. A restatement of the reference's resize_center_crop
// and compose_and_patchify (src/models/gwp05/engine/vae.cpp:1-134); compiled
// without FMA contraction so that its F32 arithmetic is the reference's, step
// for step.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "oracle.h"

namespace {

struct Taps {
  std::vector<int> index;
  std::vector<float> weight;
};

// Source taps and normalised weights of one output position p (crop included)
// along an axis of `source` pixels resized to `resized` (vae.cpp:26-42).
Taps axis_taps(int p, int source, int resized) {
  Taps t;
  const float scale = static_cast<float>(resized) / static_cast<float>(source);
  const float filter = std::max(1.0f, 1.0f / scale);
  const float center = (static_cast<float>(p) + 0.5f) / scale - 0.5f;
  const int lo = static_cast<int>(std::ceil(center - filter));
  const int hi = static_cast<int>(std::floor(center + filter));
  float sum = 0.0f;
  for (int i = lo; i <= hi; ++i) {
    const float w = std::max(0.0f, 1.0f - std::fabs(static_cast<float>(i) - center) / filter);
    if (w == 0.0f) continue;
    t.index.push_back(std::min(source - 1, std::max(0, i)));
    t.weight.push_back(w);
    sum += w;
  }
  for (float& w : t.weight) w /= sum;
  return t;
}

float pixel(const void* data, int format, int w, int x, int y, int c) {
  const size_t i = (static_cast<size_t>(y) * w + x) * 3 + c;
  return format == 0 ? static_cast<const uint8_t*>(data)[i] * (1.0f / 255.0f)
                     : static_cast<const float*>(data)[i];
}

// One view into the canvas cell [x0, x0 + cw) x [y0, y0 + ch) (vae.cpp:1-89).
void place(const void* data, int format, int sw, int sh, int cw, int ch, int x0, int y0,
           int canvas_w, std::vector<float>& canvas) {
  const float scale = std::max(static_cast<float>(cw) / sw, static_cast<float>(ch) / sh);
  const int rw = static_cast<int>(std::lround(sw * scale));
  const int rh = static_cast<int>(std::lround(sh * scale));
  const int crop_x = (rw - cw) / 2, crop_y = (rh - ch) / 2;
  std::vector<Taps> tx(cw), ty(ch);
  for (int x = 0; x < cw; ++x) tx[x] = axis_taps(x + crop_x, sw, rw);
  for (int y = 0; y < ch; ++y) ty[y] = axis_taps(y + crop_y, sh, rh);
  // Horizontal pass over every source row, then the vertical pass.
  std::vector<float> rows(static_cast<size_t>(sh) * cw * 3);
  for (int y = 0; y < sh; ++y)
    for (int x = 0; x < cw; ++x)
      for (int c = 0; c < 3; ++c) {
        float v = 0.0f;
        for (size_t i = 0; i < tx[x].index.size(); ++i)
          v += pixel(data, format, sw, tx[x].index[i], y, c) * tx[x].weight[i];
        rows[(static_cast<size_t>(y) * cw + x) * 3 + c] = v;
      }
  for (int y = 0; y < ch; ++y)
    for (int x = 0; x < cw; ++x)
      for (int c = 0; c < 3; ++c) {
        float v = 0.0f;
        for (size_t i = 0; i < ty[y].index.size(); ++i)
          v += rows[(static_cast<size_t>(ty[y].index[i]) * cw + x) * 3 + c] * ty[y].weight[i];
        canvas[(static_cast<size_t>(y0 + y) * canvas_w + x0 + x) * 3 + c] = v;
      }
}

}  // namespace

extern "C" int oracle_compose_and_patchify(const void* const* data, const int* w, const int* h,
                                           const int* format, int out_w, int out_h, float* out) {
  if (out_w <= 0 || out_h <= 0 || out_w % 2 || out_h % 2) return 1;
  for (int i = 0; i < 3; ++i)
    if (!data[i] || w[i] <= 0 || h[i] <= 0 || (format[i] != 0 && format[i] != 1)) return 1;
  const int top = out_h / 2, left = out_w / 2;
  std::vector<float> canvas(static_cast<size_t>(out_w) * out_h * 3);
  place(data[0], format[0], w[0], h[0], out_w, top, 0, 0, out_w, canvas);
  place(data[1], format[1], w[1], h[1], left, out_h - top, 0, top, out_w, canvas);
  place(data[2], format[2], w[2], h[2], out_w - left, out_h - top, left, top, out_w, canvas);
  // Patchify 2x2: packed channel (c * 2 + dx) * 2 + dy (vae.cpp:117-132).
  const int pw = out_w / 2, ph = out_h / 2;
  for (int c = 0; c < 3; ++c)
    for (int dx = 0; dx < 2; ++dx)
      for (int dy = 0; dy < 2; ++dy)
        for (int y = 0; y < ph; ++y)
          for (int x = 0; x < pw; ++x) {
            const float v = canvas[(static_cast<size_t>(2 * y + dy) * out_w + 2 * x + dx) * 3 + c];
            out[(static_cast<size_t>((c * 2 + dx) * 2 + dy) * ph + y) * pw + x] = v * 2.0f - 1.0f;
          }
  return 0;
}
