"""wam_b200_op_gemm_noalloc: the split-K GEMM for callers that cannot allocate.

Some callers of this library must not call cudaMalloc: a robot control loop
that runs the policy every cycle cannot afford the device-wide synchronization
and unbounded latency an allocation may cause, and a host framework that owns
the device allocator may forbid side allocations. This entry point runs the
same GEMM with its split-K scratch in a fixed, library-owned device array.

Checked here through the C ABI: its output matches the existing entry point
(wam_b200_op_gemm) within the GEMM tests' tolerance (raw F32 accumulators
within 1e-5 relative-L2, BF16 epilogue outputs within 1e-2) on two calls in a
row (the second call reuses the array's leftover contents), and shapes beyond
the array's size are rejected. This file is collected last so that a run that
stops at the first failure has already run every other test.
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


@pytest.mark.parametrize("m,n,k,splits,epi", [
    (48, 3072, 3072, 0, 6),     # batch-1 denoise projection, automatic split-K, F32 out
    (48, 3072, 3072, 3, 6),     # a split count clusters cannot take
    (48, 768, 1024, 7, 0),      # BF16 output with bias
])
def test_noalloc_matches_workspace_gemm_twice(cuda_device, m, n, k, splits, epi):
    import wam_b200
    from wam_b200 import ops

    lib = wam_b200.load()
    g = torch.Generator(device="cpu").manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    dt = torch.float32 if epi == 6 else torch.bfloat16
    ref = ops.gemm(x, w, epi, bias=b, scratch=ops.Scratch(), force_splits=splits)
    tol = 1e-5 if epi == 6 else 1e-2
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        rc = _noalloc(lib, x, w, epi, b, out, splits)
        assert rc == 0, wam_b200.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_l2(out.float(), ref.float()) < tol


def test_noalloc_rejects_oversized_split(cuda_device):
    import wam_b200

    lib = wam_b200.load()
    x = torch.zeros(768, 3072, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(3072, 3072, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(768, 3072, dtype=torch.float32, device="cuda")
    rc = _noalloc(lib, x, w, 6, None, out, 8)
    assert rc != 0
    assert "scratch holds" in wam_b200.last_error()
