// C ABI of the vision front-end (include/wam_b200.h, "vision"): the
// preprocessor object of the reference's cuda_preprocess.{h,cu} and the
// device-resident op form.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "c_api_util.h"
#include "kernels.h"
#include "wam_b200.h"

struct wam_b200_preprocessor {
  int device = 0;
  void* images[3] = {nullptr, nullptr, nullptr};
  size_t capacity[3] = {0, 0, 0};
};

namespace {

int vfail(wam_b200_status* st, int code, const std::string& msg) {
  wamb::set_last_error(msg);
  if (st) {
    st->code = code;
    st->message = static_cast<char*>(std::malloc(msg.size() + 1));
    if (st->message) std::memcpy(st->message, msg.c_str(), msg.size() + 1);
  }
  return code;
}

int vok(wam_b200_status* st) {
  if (st) {
    st->code = WAM_B200_OK;
    st->message = nullptr;
  }
  return WAM_B200_OK;
}

// The reference's argument checks (cuda_preprocess.cu:153-165), plus even
// output sides (the 2x2 patchify and the half-canvas split need them).
std::string check_views(const wam_b200_image* images, int count, int out_w, int out_h) {
  if (!images || count != 3) return "exactly three input images are required";
  if (out_w <= 0 || out_h <= 0 || out_w % 2 || out_h % 2)
    return "output width and height must be positive and even";
  if (static_cast<long long>(out_w / 2) * (out_h / 2) > (1ll << 30)) return "output is too large";
  for (int i = 0; i < 3; ++i) {
    const wam_b200_image& im = images[i];
    if (!im.data || im.w <= 0 || im.h <= 0) return "invalid image " + std::to_string(i);
    if (im.format != WAM_B200_PIXEL_U8 && im.format != WAM_B200_PIXEL_F32_RGB_01)
      return "image " + std::to_string(i) + ": unsupported pixel format";
    if (static_cast<long long>(im.w) * im.h > (1ll << 30))
      return "image " + std::to_string(i) + " is too large";
  }
  return "";
}

size_t view_bytes(const wam_b200_image& im) {
  return static_cast<size_t>(im.w) * im.h * 3 * (im.format == WAM_B200_PIXEL_U8 ? 1 : 4);
}

}  // namespace

extern "C" {

WAM_B200_API int wam_b200_preprocessor_create(int device_index, wam_b200_preprocessor** out,
                                              wam_b200_status* st) {
  if (!out) return vfail(st, WAM_B200_INVALID_ARGUMENT, "preprocessor pointer is required");
  *out = nullptr;
  if (cudaSetDevice(device_index) != cudaSuccess)
    return vfail(st, WAM_B200_CUDA_ERROR, "cudaSetDevice(" + std::to_string(device_index) + ") failed");
  std::string why;
  const int rc = wamb::check_sm100(&why);
  if (rc != WAM_B200_OK) return vfail(st, rc, why);
  auto* p = new wam_b200_preprocessor();
  p->device = device_index;
  *out = p;
  return vok(st);
}

WAM_B200_API void wam_b200_preprocessor_destroy(wam_b200_preprocessor* p) {
  if (!p) return;
  cudaSetDevice(p->device);
  for (void* im : p->images) cudaFree(im);
  delete p;
}

WAM_B200_API int wam_b200_preprocess(wam_b200_preprocessor* p, const wam_b200_image* images,
                                     int image_count, int out_w, int out_h, float* out,
                                     void* stream, wam_b200_status* st) {
  if (!p || !out) return vfail(st, WAM_B200_INVALID_ARGUMENT, "preprocessor and output are required");
  const std::string bad = check_views(images, image_count, out_w, out_h);
  if (!bad.empty()) return vfail(st, WAM_B200_INVALID_ARGUMENT, bad);
  if (cudaSetDevice(p->device) != cudaSuccess)
    return vfail(st, WAM_B200_CUDA_ERROR, "cudaSetDevice failed");
  auto s = static_cast<cudaStream_t>(stream);
  wamb::PreprocessView views[3];
  for (int i = 0; i < 3; ++i) {
    const size_t bytes = view_bytes(images[i]);
    if (bytes > p->capacity[i]) {
      cudaFree(p->images[i]);
      p->images[i] = nullptr;
      p->capacity[i] = 0;
      if (cudaMalloc(&p->images[i], bytes) != cudaSuccess)
        return vfail(st, WAM_B200_CUDA_ERROR, "image buffer allocation failed");
      p->capacity[i] = bytes;
    }
    if (cudaMemcpyAsync(p->images[i], images[i].data, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
      return vfail(st, WAM_B200_CUDA_ERROR, "image upload failed");
    views[i] = wamb::PreprocessView{p->images[i], images[i].w, images[i].h, images[i].format};
  }
  if (!wamb::launch_preprocess(views, out_w, out_h, out, s))
    return vfail(st, WAM_B200_CUDA_ERROR, "preprocess kernel launch failed");
  const cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return vfail(st, WAM_B200_CUDA_ERROR, cudaGetErrorString(e));
  return vok(st);
}

WAM_B200_API int wam_b200_op_preprocess(const wam_b200_image* images, int out_w, int out_h,
                                        float* out, void* stream) {
  if (!out) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "output is required");
  const std::string bad = check_views(images, 3, out_w, out_h);
  if (!bad.empty()) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, bad);
  wamb::PreprocessView views[3];
  for (int i = 0; i < 3; ++i)
    views[i] = wamb::PreprocessView{images[i].data, images[i].w, images[i].h, images[i].format};
  if (!wamb::launch_preprocess(views, out_w, out_h, out, static_cast<cudaStream_t>(stream)))
    return vfail(nullptr, WAM_B200_CUDA_ERROR, "preprocess kernel launch failed");
  return WAM_B200_OK;
}

}  // extern "C"
