// C ABI of the vision front-end (include/wam_b200.h, "vision"): the
// preprocessor object of the reference's cuda_preprocess.{h,cu} and the
// device-resident op form.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "c_api_util.h"
#include "kernels.h"
#include "vae.h"
#include "wam_b200.h"

struct wam_b200_preprocessor {
  int device = 0;
  void* images[3] = {nullptr, nullptr, nullptr};
  size_t capacity[3] = {0, 0, 0};
};

struct wam_b200_vae {
  wamb::VaeEncoder enc;
  int device = 0;
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

WAM_B200_API int wam_b200_conv_cin_pad(int cin) { return wamb::conv_cin_pad(cin); }
WAM_B200_API int wam_b200_conv_cout_pad(int cout) { return wamb::conv_cout_pad(cout); }

WAM_B200_API int wam_b200_op_conv_weight_layout(const void* src, void* dst, int cout, int cin,
                                                int taps, void* stream) {
  if (!src || !dst || cout <= 0 || cin <= 0 || (taps != 1 && taps != 9))
    return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "conv weight layout: bad arguments");
  wamb::launch_conv_weight_layout(static_cast<const wamb::bf16*>(src), static_cast<wamb::bf16*>(dst),
                                  cout, cin, taps, static_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess
             ? WAM_B200_OK
             : vfail(nullptr, WAM_B200_CUDA_ERROR, "conv weight layout launch failed");
}

WAM_B200_API int wam_b200_op_conv2d(const void* x, int in_w, int in_h, int cin, int mode,
                                    const void* w_laid, int cout, int epilogue, const void* bias,
                                    const void* residual, void* out, unsigned* error,
                                    void* stream) {
  std::string why;
  const int rc = wamb::check_sm100(&why);
  if (rc != WAM_B200_OK) return vfail(nullptr, rc, why);
  if (!x || !w_laid || !out || !error)
    return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "conv: x, weights, out and error are required");
  wamb::ConvOp op;
  const char* err = wamb::conv_plan(&op, static_cast<const wamb::bf16*>(x), in_w, in_h, cin, mode,
                                    static_cast<const wamb::bf16*>(w_laid), cout, epilogue,
                                    static_cast<const wamb::bf16*>(bias),
                                    static_cast<const wamb::bf16*>(residual),
                                    static_cast<wamb::bf16*>(out), wamb::num_sms_current());
  if (err) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, err);
  if (!wamb::conv_launch(op, error, static_cast<cudaStream_t>(stream), false))
    return vfail(nullptr, WAM_B200_CUDA_ERROR, "conv launch failed");
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_vae_tensor_spec(int z_dim, int index, char* name, size_t name_n,
                                          long long* shape4) {
  const auto specs = wamb::vae_tensor_specs(z_dim);
  if (index < 0 || index >= static_cast<int>(specs.size()) || !name || name_n == 0) return -1;
  const auto& s = specs[static_cast<size_t>(index)];
  std::snprintf(name, name_n, "%s", s.first.c_str());
  for (size_t i = 0; i < 4; ++i) shape4[i] = i < s.second.size() ? s.second[i] : 0;
  return static_cast<int>(s.second.size());
}

WAM_B200_API int wam_b200_vae_create(const wam_b200_vae_options* o, wam_b200_vae** out,
                                     wam_b200_status* st) {
  if (!o || !out) return vfail(st, WAM_B200_INVALID_ARGUMENT, "options and VAE pointer are required");
  *out = nullptr;
  if (o->struct_size < sizeof(wam_b200_vae_options))
    return vfail(st, WAM_B200_INVALID_ARGUMENT, "wam_b200_vae_options.struct_size is too small");
  if (cudaSetDevice(o->device_index) != cudaSuccess)
    return vfail(st, WAM_B200_CUDA_ERROR, "cudaSetDevice failed");
  std::string why;
  const int rc = wamb::check_sm100(&why);
  if (rc != WAM_B200_OK) return vfail(st, rc, why);
  wamb::VaeOptions vo;
  vo.artifact_path = o->artifact_path ? o->artifact_path : "";
  vo.synthetic_seed = o->synthetic_seed;
  vo.image_width = o->image_width;
  vo.image_height = o->image_height;
  vo.z_dim = o->z_dim;
  vo.device_index = o->device_index;
  vo.use_cuda_graph = o->use_cuda_graph != 0;
  auto* v = new wam_b200_vae();
  v->device = o->device_index;
  std::string err;
  if (!v->enc.init(vo, &err)) {
    delete v;
    return vfail(st, WAM_B200_INVALID_ARGUMENT, err);
  }
  *out = v;
  return vok(st);
}

WAM_B200_API void wam_b200_vae_destroy(wam_b200_vae* v) {
  if (!v) return;
  cudaSetDevice(v->device);
  delete v;
}

WAM_B200_API int wam_b200_vae_info(const wam_b200_vae* v, int* latent_count, int* launches,
                                   double* flops) {
  if (!v) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "VAE is required");
  if (latent_count) *latent_count = v->enc.latent_count();
  if (launches) *launches = v->enc.launches();
  if (flops) *flops = v->enc.flops();
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_vae_encode_device(wam_b200_vae* v, const float* pixels, float* latent,
                                            void* stream, wam_b200_status* st) {
  if (!v || !pixels || !latent)
    return vfail(st, WAM_B200_INVALID_ARGUMENT, "VAE, pixels and latent are required");
  std::string err;
  if (!v->enc.encode(pixels, latent, static_cast<cudaStream_t>(stream), &err))
    return vfail(st, WAM_B200_CUDA_ERROR, err);
  return vok(st);
}

WAM_B200_API int wam_b200_vae_encode(wam_b200_vae* v, const wam_b200_image* images,
                                     int image_count, float* latent, size_t latent_n,
                                     wam_b200_status* st) {
  if (!v || !latent) return vfail(st, WAM_B200_INVALID_ARGUMENT, "VAE and latent are required");
  const auto& o = v->enc.options();
  if (latent_n != static_cast<size_t>(v->enc.latent_count()))
    return vfail(st, WAM_B200_INVALID_ARGUMENT,
                 "latent buffer must hold z_dim * (H / 16) * (W / 16) = " +
                     std::to_string(v->enc.latent_count()) + " floats");
  cudaStream_t s = v->enc.stream();
  const std::string bad = check_views(images, image_count, o.image_width, o.image_height);
  if (!bad.empty()) return vfail(st, WAM_B200_INVALID_ARGUMENT, bad);
  wamb::PreprocessView views[3];
  for (int i = 0; i < 3; ++i)
    views[i] = wamb::PreprocessView{images[i].data, images[i].w, images[i].h, images[i].format};
  std::string err;
  if (!v->enc.encode_images(views, 3, v->enc.latent_slot(), s, &err))
    return vfail(st, WAM_B200_CUDA_ERROR, err);
  if (cudaMemcpyAsync(latent, v->enc.latent_slot(), latent_n * sizeof(float),
                      cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return vfail(st, WAM_B200_CUDA_ERROR, "latent readback failed");
  const cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return vfail(st, WAM_B200_CUDA_ERROR, cudaGetErrorString(e));
  unsigned word = 0;
  cudaMemcpy(&word, v->enc.error_word(), sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (word) return vfail(st, WAM_B200_CUDA_ERROR, "VAE kernel wait timed out (device error word set)");
  return vok(st);
}

WAM_B200_API int wam_b200_vae_read_stage(wam_b200_vae* v, const char* name, float* out, size_t n,
                                         int* h, int* w, int* c) {
  if (!v || !name || !out) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "bad arguments");
  std::vector<float> buf;
  int hh = 0, ww = 0, cc = 0;
  cudaStreamSynchronize(v->enc.stream());
  if (!v->enc.read_stage(name, &buf, &hh, &ww, &cc))
    return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, std::string("no VAE stage ") + name);
  if (buf.size() > n) return vfail(nullptr, WAM_B200_INVALID_ARGUMENT, "stage buffer too small");
  std::memcpy(out, buf.data(), buf.size() * sizeof(float));
  if (h) *h = hh;
  if (w) *w = ww;
  if (c) *c = cc;
  return WAM_B200_OK;
}

}  // extern "C"
