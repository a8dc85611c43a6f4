"""ctypes structures and prototypes of the engine-level C ABI (include/wam_b200.h)."""
from __future__ import annotations

import ctypes as C

GEOM_FIELDS = ("hidden", "layers", "heads", "ffn", "action_hidden", "action_ffn", "action_dim",
               "real_state_dim", "real_action_dim", "num_embodiments", "embodiment_id", "grid_h",
               "grid_w", "vae_z", "action_chunk", "steps", "prompt_tokens", "text_dim")


class Status(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_void_p)]


class Geometry(C.Structure):
    _fields_ = [(n, C.c_int) for n in GEOM_FIELDS] + [("norm_eps", C.c_float),
                                                      ("flow_shift", C.c_float)]


class Options(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("artifact_path", C.c_char_p),
                ("synthetic_geometry", Geometry), ("synthetic_seed", C.c_uint64),
                ("synthetic_bias_scale", C.c_float), ("device_index", C.c_int),
                ("max_batch", C.c_int), ("use_cuda_graphs", C.c_int), ("prompt_cache", C.c_int),
                ("weight_format", C.c_int), ("ffn_kind", C.c_int), ("norm_kind", C.c_int),
                ("block_mode", C.c_int), ("vae", C.c_int), ("t5", C.c_int),
                ("t5_vocab", C.c_int), ("t5_ffn", C.c_int), ("t5_layers", C.c_int)]


class Image(C.Structure):
    _fields_ = [("data", C.c_void_p), ("w", C.c_int), ("h", C.c_int), ("format", C.c_int)]


class BlockInputs(C.Structure):
    _fields_ = [("visual", C.POINTER(C.c_float)), ("action", C.POINTER(C.c_float)),
                ("text_visual", C.POINTER(C.c_float)), ("text_action", C.POINTER(C.c_float)),
                ("timestep", C.c_float)]


class Request(C.Structure):
    _fields_ = [("state", C.POINTER(C.c_float)), ("state_n", C.c_int),
                ("noise", C.POINTER(C.c_float)), ("ref_latent", C.POINTER(C.c_float)),
                ("ref_latent_n", C.c_longlong), ("prompt_emb", C.POINTER(C.c_float)),
                ("prompt_tokens", C.c_int), ("images", C.POINTER(Image)), ("n_images", C.c_int),
                ("lang_tokens", C.POINTER(C.c_int32)), ("n_lang", C.c_int),
                ("attention_mask", C.POINTER(C.c_int32)), ("attention_mask_n", C.c_int)]


class Stats(C.Structure):
    _fields_ = [("ms_total", C.c_float), ("ms_device", C.c_float), ("prompt_cache_hit", C.c_int),
                ("kernel_launches", C.c_int), ("resident_device_bytes", C.c_uint64)]


class OpProfile(C.Structure):
    _fields_ = [("phase", C.c_int), ("kind", C.c_int), ("launches", C.c_int), ("ms", C.c_float),
                ("bytes", C.c_double), ("flops", C.c_double), ("shape", C.c_int * 4)]


class GraphProfile(C.Structure):
    _fields_ = [("ms", C.c_float), ("bytes", C.c_double), ("flops", C.c_double),
                ("launches", C.c_int)]


def attach(lib, sig) -> None:
    vp, i32, sz = C.c_void_p, C.c_int, C.c_size_t
    f32p = C.POINTER(C.c_float)
    st = C.POINTER(Status)
    sig(lib, "wam_b200_status_free", None, [st])
    sig(lib, "wam_b200_create", i32, [C.POINTER(Options), C.POINTER(vp), st])
    sig(lib, "wam_b200_destroy", None, [vp])
    sig(lib, "wam_b200_reset", i32, [vp])
    sig(lib, "wam_b200_geometry_of", i32, [vp, C.POINTER(Geometry)])
    sig(lib, "wam_b200_max_batch", i32, [vp])
    sig(lib, "wam_b200_batcher_create", i32, [vp, i32, C.POINTER(vp), st])
    sig(lib, "wam_b200_batcher_destroy", None, [vp])
    sig(lib, "wam_b200_batcher_predict", i32, [vp, C.POINTER(Request), f32p, sz,
                                               C.POINTER(Stats), C.POINTER(i32), st])
    sig(lib, "wam_b200_batcher_counts", i32, [vp, C.POINTER(C.c_longlong),
                                              C.POINTER(C.c_longlong)])
    sig(lib, "wam_b200_predict", i32, [vp, C.POINTER(Request), f32p, sz, C.POINTER(Stats), st])
    sig(lib, "wam_b200_predict_batch", i32,
        [vp, C.POINTER(Request), i32, f32p, sz, C.POINTER(Stats), st])
    sig(lib, "wam_b200_stage", i32, [vp, C.POINTER(Request), i32, st])
    sig(lib, "wam_b200_run", i32, [vp, i32, st])
    sig(lib, "wam_b200_fetch", i32, [vp, C.POINTER(Request), i32, f32p, sz, st])
    sig(lib, "wam_b200_stream", vp, [vp])
    sig(lib, "wam_b200_kernel_launches", i32, [vp, i32, i32])
    sig(lib, "wam_b200_read_tensor", i32, [vp, C.c_char_p, i32, i32, f32p, sz, st])
    sig(lib, "wam_b200_phase_ms", i32, [vp, f32p, f32p, f32p])
    sig(lib, "wam_b200_profile", i32, [vp, i32, C.POINTER(OpProfile), i32, st])
    sig(lib, "wam_b200_profile_graph", i32, [vp, i32, i32, i32, i32, C.POINTER(GraphProfile), st])
    sig(lib, "wam_b200_profile_graph_lane", i32,
        [vp, i32, i32, i32, i32, i32, C.POINTER(GraphProfile), st])
    sig(lib, "wam_b200_block_forward", i32,
        [vp, C.POINTER(BlockInputs), f32p, sz, f32p, sz, f32p, st])
