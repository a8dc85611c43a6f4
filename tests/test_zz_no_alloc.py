"""wam_b200_op_gemm_noalloc: the split-K GEMM for callers that cannot allocate.

Some callers of this library must not call cudaMalloc: a robot control loop
that runs the policy every cycle cannot afford the device-wide synchronization
and unbounded latency an allocation may cause, and a host framework that owns
the device allocator may forbid side allocations. This entry point runs the
same GEMM with its split-K scratch in a fixed, library-owned device array.

Checked here through the C ABI, on two calls in a row (the second call reuses
the array's leftover contents: its tile counters and error word):
  * the output matches the existing entry point (wam_b200_op_gemm with a
    caller workspace) within the GEMM tests' tolerance (raw F32 accumulators
    within 1e-5 relative-L2, BF16 epilogue outputs within 1e-2) and an
    independent F32 matmul of the same BF16 operands within 1e-2;
  * the error word reads 0 after every call;
  * a split count above 8 (tile counters, the last CTA of a tile reduces),
    and an unsplit shape with more output tiles than the array has counters,
    both run; a split-K shape whose partials exceed the array is rejected.
This file is collected last so that a run that stops at the first failure has
already run every other test.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _noalloc(lib, x, w, epi, bias, out, splits):
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.wam_b200_op_gemm_noalloc(_p(x), x.stride(0), x.shape[0], _p(w), w.shape[0],
                                        w.shape[1], epi, _p(bias), None, None, 0, _p(out),
                                        out.stride(0), splits, s)


def _error_word(lib):
    code = C.c_uint(0xFFFFFFFF)
    assert lib.wam_b200_op_gemm_noalloc_error(C.byref(code)) == 0
    return code.value


def _f32_reference(x, w, b, epi):
    acc = x.float() @ w.float().T
    if epi == 6:
        return acc
    # EPI_BIAS: bf16(bf16(acc) + b)
    return (acc.to(torch.bfloat16).float() + b.float()).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k,splits,epi", [
    (48, 3072, 3072, 0, 6),     # batch-1 denoise projection, automatic split-K, F32 out
    (48, 3072, 3072, 3, 6),     # a split count clusters cannot take
    (48, 3072, 3072, 12, 6),    # > 8 splits: tile counters, the last CTA reduces
    (48, 768, 1024, 7, 0),      # BF16 output with bias
])
def test_noalloc_matches_workspace_gemm_twice(cuda_device, m, n, k, splits, epi):
    import wam_b200
    from wam_b200 import ops

    lib = wam_b200.load()
    g = torch.Generator(device="cpu").manual_seed(m + n + k + splits)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    dt = torch.float32 if epi == 6 else torch.bfloat16
    ref = ops.gemm(x, w, epi, bias=b, scratch=ops.Scratch(), force_splits=splits)
    f32 = _f32_reference(x, w, b, epi)
    tol = 1e-5 if epi == 6 else 1e-2
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        rc = _noalloc(lib, x, w, epi, b, out, splits)
        assert rc == 0, wam_b200.last_error()
        torch.cuda.synchronize()
        assert _error_word(lib) == 0
        assert torch.isfinite(out.float()).all()
        assert rel_l2(out.float(), ref.float()) < tol
        assert rel_l2(out.float(), f32.float()) < 1e-2


def test_noalloc_large_unsplit_shape(cuda_device):
    """Batch-64 prefix shape: 384 x 12 = 4608 output tiles (more than the
    array's 4096 tile counters) but unsplit and persistent, so it needs none
    of the array's partials or counters."""
    import wam_b200

    lib = wam_b200.load()
    g = torch.Generator(device="cpu").manual_seed(5)
    m, n, k = 49152, 3072, 3072
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    ref = _f32_reference(x, w, b, 0)
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _noalloc(lib, x, w, 0, b, out, 0)
        assert rc == 0, wam_b200.last_error()
        torch.cuda.synchronize()
        assert _error_word(lib) == 0
        assert rel_l2(out.float(), ref.float()) < 1e-2


def test_noalloc_rejects_oversized_split(cuda_device):
    import wam_b200

    lib = wam_b200.load()
    x = torch.zeros(768, 3072, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(3072, 3072, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(768, 3072, dtype=torch.float32, device="cuda")
    rc = _noalloc(lib, x, w, 6, None, out, 8)
    assert rc != 0
    assert "scratch holds" in wam_b200.last_error()
