"""Op-level wrappers over the C ABI, taking torch CUDA tensors.

torch supplies device memory and the current stream only; the arithmetic runs
in libwam_b200's sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import check, load

(EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_SILU, EPI_GATED_RES, EPI_RES, EPI_F32_BIAS, EPI_F32_OUT,
 EPI_BIAS_GELU_R, EPI_BIAS_GELU_ERF, EPI_MUL) = range(10)


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class Scratch:
    """Split-K workspace + counters + device error word for op-level GEMMs."""

    def __init__(self, floats: int = 1 << 24, slots: int = 1 << 14, device="cuda"):
        self.ws = torch.zeros(floats, dtype=torch.float32, device=device)
        self.counters = torch.zeros(slots, dtype=torch.int32, device=device)
        self.error = torch.zeros(1, dtype=torch.int32, device=device)

    def error_code(self) -> int:
        return int(self.error.item())


_error_words = {}


GEMM_TILED_WEIGHTS = 0x100


class TiledWeight:
    """A [n, k] BF16 weight re-tiled by wam_b200_op_retile_weights into
    contiguous 16 KB UMMA tiles; `data` is the flat device buffer."""

    def __init__(self, w):
        n, k = w.shape
        self.shape = (n, k)
        self.device = w.device
        self.data = torch.empty(n * k, dtype=torch.bfloat16, device=w.device)
        w = w.contiguous()
        rc = load().wam_b200_op_retile_weights(_ptr(w), _ptr(self.data), n, k, _stream())
        check(rc, "wam_b200_op_retile_weights")


GEMM_Q8_WEIGHTS = 0x200
GEMM_PAIR = 0x400  # CTA-pair (cta_group::2) kernel for >= 256 token rows
Q8_TILE_BYTES = 256 * 64 + 256 * 2 * 2


def q8_quantize(w, out=None):
    """BF16 [n, k] -> GGML Q8_0 blocks (uint8 [n * k / 32, 34]) on the device."""
    w = w.contiguous()
    if out is None:
        out = torch.empty(w.numel() // 32, 34, dtype=torch.uint8, device=w.device)
    check(load().wam_b200_op_q8_quantize(_ptr(w), w.numel(), _ptr(out), _stream()),
          "wam_b200_op_q8_quantize")
    return out


class Q8Weight:
    """A [n, k] weight as Q8_0 GEMM tiles (quantised on the device from BF16,
    or from given Q8_0 blocks); `data` holds [n/256][k/64] tiles of 17408 bytes."""

    def __init__(self, w=None, blocks=None, shape=None):
        if blocks is None:
            n, k = w.shape
            blocks = q8_quantize(w)
            device = w.device
        else:
            n, k = shape
            device = blocks.device
        self.shape = (n, k)
        self.device = device
        self.blocks = blocks
        self.data = torch.empty((n // 256) * (k // 64) * Q8_TILE_BYTES, dtype=torch.uint8, device=device)
        check(load().wam_b200_op_q8_retile(_ptr(blocks), _ptr(self.data), n, k, _stream()),
              "wam_b200_op_q8_retile")


def gemm(x, w, epilogue=EPI_BIAS, bias=None, gate=None, residual=None, out=None,
         scratch: Scratch | None = None, force_splits: int = 0, pair: bool = False):
    """out[m, n] = epilogue(x[m, :K] . w[n, :]) via wam_b200_op_gemm.

    Without `scratch`, split-K partials are reduced inside thread-block
    clusters (splits 1/2/4/8); with it, through its global workspace. `w` is a
    row-major [n, k] tensor or a TiledWeight."""
    lib = load()
    m = x.shape[0]
    n, k = w.shape
    if pair:
        epilogue |= GEMM_PAIR
    if isinstance(w, TiledWeight):
        epilogue |= GEMM_TILED_WEIGHTS
        w = w.data
    elif isinstance(w, Q8Weight):
        epilogue |= GEMM_Q8_WEIGHTS
        w = w.data
    if out is None:
        dt = torch.float32 if (epilogue & 0xFF) == EPI_F32_OUT else torch.bfloat16
        out = torch.empty(m, n, dtype=dt, device=x.device)
    if scratch is None:
        err = _error_words.setdefault(x.device, torch.zeros(1, dtype=torch.int32, device=x.device))
        ws = (C.c_void_p(0), 0, C.c_void_p(0), 0, _ptr(err))
    else:
        ws = (_ptr(scratch.ws), scratch.ws.numel(), _ptr(scratch.counters),
              scratch.counters.numel(), _ptr(scratch.error))
    rc = lib.wam_b200_op_gemm(
        _ptr(x), x.stride(0), m, _ptr(w), n, k, epilogue, _ptr(bias), _ptr(gate), _ptr(residual),
        residual.stride(0) if residual is not None else 0, _ptr(out), out.stride(0),
        *ws, force_splits, _stream())
    check(rc, "wam_b200_op_gemm")
    return out


def attention(q, k, v, scale=None, out=None):
    """q: [B, heads, lq, 128], k/v: [B, heads, lk, 128] BF16 (contiguous).
    Returns [B * lq, heads * 128] BF16."""
    lib = load()
    B, heads, lq, d = q.shape
    lk = k.shape[2]
    assert d == 128 and q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
    if out is None:
        out = torch.empty(B * lq, heads * 128, dtype=torch.bfloat16, device=q.device)
    scale = scale if scale is not None else 1.0 / 128 ** 0.5
    rc = lib.wam_b200_op_attention(_ptr(q), heads * lq * 128, lq * 128, _ptr(k), _ptr(v),
                                   heads * lk * 128, lk * 128, lq, lk, heads, B, scale, _ptr(out),
                                   out.stride(0), _stream())
    check(rc, "wam_b200_op_attention")
    return out


def layernorm(x, a, b, eps=1e-6, affine=False, out=None):
    lib = load()
    y = torch.empty_like(x) if out is None else out
    rc = lib.wam_b200_op_layernorm(_ptr(x), x.shape[0], x.shape[1], _ptr(a), _ptr(b), eps,
                                   1 if affine else 0, _ptr(y), _stream())
    check(rc, "wam_b200_op_layernorm")
    return y


def synth(n, seed, name, scale, center, device="cuda"):
    lib = load()
    w = torch.empty(n, dtype=torch.bfloat16, device=device)
    ts = lib.wam_b200_tensor_seed(seed, name.encode())
    rc = lib.wam_b200_op_synth(_ptr(w), n, ts, scale, center, _stream())
    check(rc, "wam_b200_op_synth")
    return w


class QkvScatterArgs(C.Structure):
    """wam_b200_qkv_scatter_args (include/wam_b200.h)."""

    _fields_ = [("src", C.c_void_p), ("ld_src", C.c_int), ("rows", C.c_int),
                ("rows_per_seq", C.c_int), ("heads", C.c_int), ("q_col", C.c_int),
                ("k_col", C.c_int), ("v_col", C.c_int), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p), ("eps", C.c_float), ("rope_mode", C.c_int),
                ("pos_base", C.c_int), ("pos_thw", C.c_void_p), ("inv_freq", C.c_void_p),
                ("q_out", C.c_void_p), ("q_seq_stride", C.c_longlong),
                ("q_head_stride", C.c_longlong), ("q_row_offset", C.c_int),
                ("k_out", C.c_void_p), ("v_out", C.c_void_p), ("kv_seq_stride", C.c_longlong),
                ("kv_head_stride", C.c_longlong), ("kv_row_offset", C.c_int)]


def rope_inv_freq(mode: int, device="cuda"):
    """RoPE inverse frequencies [64] of wam_b200_rope_inv_freq, on the device."""
    buf = (C.c_float * 64)()
    check(load().wam_b200_rope_inv_freq(mode, buf), "wam_b200_rope_inv_freq")
    return torch.tensor(list(buf), dtype=torch.float32, device=device)


def qkv_scatter(src, heads, rows_per_seq, q_out=None, k_out=None, v_out=None, q_norm=None,
                k_norm=None, eps=1e-6, rope_mode=0, pos_base=0, pos_thw=None, q_row_offset=0,
                kv_row_offset=0, cols=(0, None, None)):
    """src: [rows, ld] BF16 packed projection; q_out: [B, heads, Rq, 128],
    k_out / v_out: [B, heads, Rkv, 128] BF16 caches (written at the row offsets).
    cols: first source column of (q, k, v); None skips a part."""
    H = heads * 128
    a = QkvScatterArgs()
    a.src = src.data_ptr()
    a.ld_src = src.stride(0)
    a.rows = src.shape[0]
    a.rows_per_seq = rows_per_seq
    a.heads = heads
    qc, kc, vc = cols
    a.q_col = -1 if qc is None else qc
    a.k_col = -1 if kc is None else kc
    a.v_col = -1 if vc is None else vc
    a.q_norm = q_norm.data_ptr() if q_norm is not None else None
    a.k_norm = k_norm.data_ptr() if k_norm is not None else None
    a.eps = eps
    a.rope_mode = rope_mode
    a.pos_base = pos_base
    keep = []
    if rope_mode:
        inv = rope_inv_freq(rope_mode, src.device)
        keep.append(inv)
        a.inv_freq = inv.data_ptr()
    if pos_thw is not None:
        a.pos_thw = pos_thw.data_ptr()
    if q_out is not None:
        a.q_out = q_out.data_ptr()
        a.q_seq_stride = q_out.stride(0)
        a.q_head_stride = q_out.stride(1)
    a.q_row_offset = q_row_offset
    kv = k_out if k_out is not None else v_out
    if k_out is not None:
        a.k_out = k_out.data_ptr()
    if v_out is not None:
        a.v_out = v_out.data_ptr()
    if kv is not None:
        a.kv_seq_stride = kv.stride(0)
        a.kv_head_stride = kv.stride(1)
    a.kv_row_offset = kv_row_offset
    assert H <= src.shape[1]
    rc = load().wam_b200_op_qkv_scatter(C.byref(a), _stream())
    check(rc, "wam_b200_op_qkv_scatter")
    torch.cuda.current_stream().synchronize() if keep else None


CONV_3X3, CONV_3X3_S2, CONV_1X1 = 0, 1, 2


class ConvWeight:
    """A [cout, cin, kh, kw] BF16 convolution weight laid out for the implicit-
    GEMM kernel by wam_b200_op_conv_weight_layout: [cout_pad][taps][cin_pad]."""

    def __init__(self, w):
        lib = load()
        _conv_sigs(lib)
        cout, cin, kh, kw = w.shape
        taps = kh * kw
        if (kh, kw) not in ((3, 3), (1, 1)):
            raise ValueError("conv kernels are 3x3 or 1x1")
        self.cout, self.cin, self.taps = cout, cin, taps
        self.data = torch.empty(lib.wam_b200_conv_cout_pad(cout) * taps *
                                lib.wam_b200_conv_cin_pad(cin), dtype=torch.bfloat16,
                                device=w.device)
        rc = lib.wam_b200_op_conv_weight_layout(_ptr(w.contiguous()), _ptr(self.data), cout, cin,
                                                taps, _stream())
        check(rc, "wam_b200_op_conv_weight_layout")


def _conv_sigs(lib):
    if getattr(lib, "_conv_sigs", False):
        return
    vp, i32 = C.c_void_p, C.c_int
    lib.wam_b200_conv_cin_pad.restype = i32
    lib.wam_b200_conv_cin_pad.argtypes = [i32]
    lib.wam_b200_conv_cout_pad.restype = i32
    lib.wam_b200_conv_cout_pad.argtypes = [i32]
    lib.wam_b200_op_conv_weight_layout.restype = i32
    lib.wam_b200_op_conv_weight_layout.argtypes = [vp, vp, i32, i32, i32, vp]
    lib.wam_b200_op_conv2d.restype = i32
    lib.wam_b200_op_conv2d.argtypes = [vp, i32, i32, i32, i32, vp, i32, i32, vp, vp, vp, vp, vp]
    lib._conv_sigs = True


def conv2d(x, w: ConvWeight, mode: int, bias=None, residual=None, out=None, error=None):
    """NHWC BF16 convolution x [H, W, cin] -> [H', W', cout] (mode CONV_3X3,
    CONV_3X3_S2 or CONV_1X1); with `residual` the epilogue adds it (EPI_RES)."""
    lib = load()
    _conv_sigs(lib)
    h, wd, cin = x.shape
    if cin != w.cin or (w.taps == 1) != (mode == CONV_1X1):
        raise ValueError("conv: weight does not match the input / mode")
    oh, ow = (h // 2, wd // 2) if mode == CONV_3X3_S2 else (h, wd)
    if out is None:
        out = torch.empty((oh, ow, w.cout), dtype=torch.bfloat16, device=x.device)
    if error is None:
        error = torch.zeros(1, dtype=torch.int32, device=x.device)
    rc = lib.wam_b200_op_conv2d(_ptr(x.contiguous()), wd, h, cin, mode, _ptr(w.data), w.cout,
                                EPI_RES if residual is not None else EPI_BIAS, _ptr(bias),
                                _ptr(residual), _ptr(out), _ptr(error), _stream())
    check(rc, "wam_b200_op_conv2d")
    return out
