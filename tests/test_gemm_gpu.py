"""tcgen05 GEMM parity against a torch F32 reference of the same op.

The GEMM is a floating-point kernel, so its reference is an F32 matmul of the
same BF16 operands; epilogues are checked against a torch restatement of the
reference's BF16 rounding points (weights.cpp:819-849, native-bf16.patch:79-91).
Tolerances: raw F32 accumulators within 1e-5 relative-L2 (summation order only);
BF16 outputs within 1 BF16 ulp on >99.9% of elements plus 1e-2 relative-L2.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def make(m, n, k, seed=0, dev="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    return x, w, b


SHAPES = [
    (48, 3072, 3072),   # denoise QKV-slice / O projection at batch 1 (split-K)
    (48, 256, 128),
    (1, 384, 256),      # single token (state / condition)
    (10, 1024, 256),    # condition MLP over 10 timesteps
    (200, 640, 192),    # patch embedding K
    (768, 3072, 3072),  # prefix visual tokens
    (768, 14336, 512),  # more tiles than SMs: persistent kernel
    (3072, 1024, 256),  # batched denoise shape class: persistent, 24 token tiles
    (384, 1536, 1024),  # batch-8 denoise
    (1000, 512, 640),   # ragged M
]


@pytest.mark.parametrize("mode", ["cluster", "workspace"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_f32_accumulator(cuda_device, m, n, k, mode):
    from wam_b200 import ops

    x, w, _ = make(m, n, k)
    scratch = ops.Scratch() if mode == "workspace" else None
    y = ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, scratch=scratch)
    ref = x.float() @ w.float().T
    torch.cuda.synchronize()
    assert rel_l2(y, ref) < 1e-5


@pytest.mark.parametrize("splits,mode", [(1, "cluster"), (2, "cluster"), (3, "cluster"),
                                         (4, "cluster"), (5, "cluster"), (6, "cluster"),
                                         (7, "cluster"), (8, "cluster"), (3, "workspace"),
                                         (7, "workspace"), (4, "workspace"), (12, "workspace")])
def test_gemm_forced_splits_deterministic(cuda_device, splits, mode):
    from wam_b200 import ops

    x, w, _ = make(48, 512, 1024, seed=1)
    s = ops.Scratch() if mode == "workspace" else None
    y1 = ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, scratch=s, force_splits=splits)
    y2 = ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, scratch=s, force_splits=splits)
    ref = x.float() @ w.float().T
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert rel_l2(y1, ref) < 1e-5
    if s is not None:
        assert s.error_code() == 0
        assert int(s.counters.abs().sum()) == 0


def test_gemm_cluster_rejects_more_than_8_splits(cuda_device):
    from wam_b200 import ops

    x, w, _ = make(48, 512, 1024, seed=1)
    with pytest.raises(RuntimeError, match="cluster split-K"):
        ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, force_splits=9)


def bf(x):
    return x.to(torch.bfloat16).float()


def gelu_tanh(v):
    return 0.5 * v * (1.0 + torch.tanh(0.7978845608028654 * v * (1.0 + 0.044715 * v * v)))


@pytest.mark.parametrize("m,n,k", [(48, 3072, 3072), (768, 1024, 512), (16, 384, 128)])
@pytest.mark.parametrize("epi", ["bias", "gelu", "gelu_r", "gelu_erf", "silu", "gated", "res",
                                 "f32bias", "mul"])
def test_gemm_epilogues(cuda_device, m, n, k, epi):
    from wam_b200 import ops

    x, w, b = make(m, n, k, seed=2)
    acc = x.float() @ w.float().T
    lin = bf(bf(acc) + b.float())
    gate = torch.randn(n, device="cuda") * 0.5
    resid = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    if epi == "bias":
        y = ops.gemm(x, w, ops.EPI_BIAS, bias=b)
        ref = lin
    elif epi == "gelu":
        y = ops.gemm(x, w, ops.EPI_BIAS_GELU, bias=b)
        ref = bf(gelu_tanh(bf(acc) + b.float()))
    elif epi == "gelu_r":
        y = ops.gemm(x, w, ops.EPI_BIAS_GELU_R, bias=b)
        ref = bf(gelu_tanh(lin))
    elif epi == "gelu_erf":
        y = ops.gemm(x, w, ops.EPI_BIAS_GELU_ERF, bias=b)
        ref = bf(0.5 * lin * (1.0 + torch.erf(lin / 2 ** 0.5)))
    elif epi == "silu":
        y = ops.gemm(x, w, ops.EPI_BIAS_SILU, bias=b)
        ref = bf(lin * torch.sigmoid(lin))
    elif epi == "gated":
        y = ops.gemm(x, w, ops.EPI_GATED_RES, bias=b, gate=gate, residual=resid)
        ref = bf(resid.float() + lin * gate)
    elif epi == "res":
        y = ops.gemm(x, w, ops.EPI_RES, bias=b, residual=resid)
        ref = bf(resid.float() + lin)
    elif epi == "mul":
        y = ops.gemm(x, w, ops.EPI_MUL, bias=b, residual=resid)
        ref = bf(resid.float() * lin)
    else:
        y = ops.gemm(x, w, ops.EPI_F32_BIAS, bias=b)
        ref = bf(acc + b.float())
    torch.cuda.synchronize()
    y = y.float()
    assert rel_l2(y, ref) < 1e-2
    # BF16 rounding of values whose F32 accumulators differ in the last bits can
    # flip by one ulp; anything beyond that is a real mismatch.
    ulp = torch.clamp(ref.abs(), min=1e-6) * (2.0 ** -7)
    bad = ((y - ref).abs() > 1.01 * ulp + 1e-6).float().mean().item()
    assert bad < 1e-3, f"{bad:.2e} of elements differ by more than one BF16 ulp"


def test_gemm_in_place_residual(cuda_device):
    """The gated-residual epilogue may write over its residual input."""
    from wam_b200 import ops

    x, w, b = make(48, 768, 512, seed=3)
    gate = torch.randn(768, device="cuda")
    h = torch.randn(48, 768, device="cuda").to(torch.bfloat16)
    expect = bf(h.float() + bf(bf(x.float() @ w.float().T) + b.float()) * gate)
    ops.gemm(x, w, ops.EPI_GATED_RES, bias=b, gate=gate, residual=h, out=h)
    torch.cuda.synchronize()
    assert rel_l2(h.float(), expect) < 1e-2


@pytest.mark.parametrize("m,n,k", [(48, 3072, 3072), (768, 1024, 512), (1, 512, 256),
                                   (384, 1536, 1024), (1000, 512, 640)])
@pytest.mark.parametrize("mode", ["cluster", "workspace"])
def test_gemm_tiled_weights_bit_exact(cuda_device, m, n, k, mode):
    """Re-tiled weights change only where each tile is fetched from, not the
    accumulation order: the result equals the row-major GEMM bit for bit."""
    from wam_b200 import ops

    x, w, b = make(m, n, k, seed=4)
    tw = ops.TiledWeight(w)
    s = ops.Scratch() if mode == "workspace" else None
    for epi in (ops.EPI_F32_OUT, ops.EPI_BIAS_GELU):
        y_row = ops.gemm(x, w, epi, bias=b, scratch=s)
        y_tiled = ops.gemm(x, tw, epi, bias=b, scratch=s)
        torch.cuda.synchronize()
        assert torch.equal(y_row, y_tiled)
    ref = x.float() @ w.float().T
    assert rel_l2(ops.gemm(x, tw, ops.EPI_F32_OUT).float(), ref) < 1e-5


def test_retile_layout(cuda_device):
    """Chunk c (8 BF16) of row r of tile (nt, kb) lands at chunk c ^ (r % 8) of
    that row inside the tile's contiguous 256 x 64 block."""
    from wam_b200 import ops

    n, k = 512, 192
    w = torch.arange(n * k, dtype=torch.float32).remainder(251).to(torch.bfloat16).view(n, k)
    w = w.to("cuda")
    got = ops.TiledWeight(w).data.view(n // 256, k // 64, 256, 8, 8).cpu()
    wc = w.cpu().view(n // 256, 256, k // 64, 8, 8).permute(0, 2, 1, 3, 4)  # nt, kb, r, c, e
    expect = torch.empty_like(got)
    for r in range(256):
        for c in range(8):
            expect[:, :, r, c ^ (r % 8)] = wc[:, :, r, c]
    assert torch.equal(got, expect)


def test_retile_rejects_bad_shapes(cuda_device):
    from wam_b200 import ops

    with pytest.raises(RuntimeError, match="retile"):
        ops.TiledWeight(torch.zeros(100, 64, dtype=torch.bfloat16, device="cuda"))
    x, w, _ = make(16, 256, 64)
    tw = ops.TiledWeight(w)
    tw.shape = (128, 64)  # not a whole number of 256-row tiles
    with pytest.raises(RuntimeError, match="multiple of 256"):
        ops.gemm(x[:, :64], tw, ops.EPI_F32_OUT)


PAIR_SHAPES = [
    (256, 512, 512),     # one pair tile
    (300, 768, 512),     # ragged: the second pair's odd CTA has no token rows
    (768, 3072, 3072),   # prefix O / cross projections (split over pairs with a workspace)
    (768, 3072, 14336),  # prefix FFN down (long K)
    (512, 9216, 1024),   # more pair tiles than resident pairs: persistent loop
    (1000, 512, 640),    # ragged M, 10 k-blocks
]


@pytest.mark.parametrize("layout", ["rowmajor", "tiled"])
@pytest.mark.parametrize("mode", ["cluster", "workspace"])
@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
def test_gemm_pair_matches_single_cta(cuda_device, m, n, k, mode, layout):
    """The CTA-pair (cta_group::2) kernel (pair=True, >= 256 token rows) and the
    default one-CTA plan: both against the F32 product, and the BF16
    gated-residual epilogue of both within one BF16 ulp of each other."""
    from wam_b200 import ops

    x, w, b = make(m, n, k, seed=5)
    wt = ops.TiledWeight(w) if layout == "tiled" else w
    scratch = ops.Scratch() if mode == "workspace" else None
    ref = x.float() @ w.float().T
    y_pair = ops.gemm(x, wt, epilogue=ops.EPI_F32_OUT, scratch=scratch, pair=True)
    y_one = ops.gemm(x, wt, epilogue=ops.EPI_F32_OUT, scratch=scratch)
    gate = torch.randn(n, device="cuda") * 0.5
    resid = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    g_pair = ops.gemm(x, wt, ops.EPI_GATED_RES, bias=b, gate=gate, residual=resid, scratch=scratch,
                      pair=True)
    g_one = ops.gemm(x, wt, ops.EPI_GATED_RES, bias=b, gate=gate, residual=resid, scratch=scratch)
    torch.cuda.synchronize()
    # F32 accumulation error grows with the reduction length (~sqrt(K)).
    tol = 1e-5 * max(1.0, math.sqrt(k / 4096))
    assert rel_l2(y_pair, ref) < tol
    assert rel_l2(y_one, ref) < tol
    g_pair, g_one = g_pair.float(), g_one.float()
    ulp = torch.clamp(g_one.abs(), min=1e-6) * (2.0 ** -7)
    bad = ((g_pair - g_one).abs() > 1.01 * ulp + 1e-6).float().mean().item()
    assert bad < 1e-3, f"{bad:.2e} of gated-residual outputs differ by more than one BF16 ulp"
    if scratch is not None:
        assert scratch.error_code() == 0


def test_gemm_pair_repeat_deterministic(cuda_device):
    """Split-over-pairs reduction runs in split order: repeated launches agree bit for bit."""
    from wam_b200 import ops

    x, w, _ = make(768, 3072, 3072, seed=6)
    s = ops.Scratch()
    y1 = ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, scratch=s, pair=True)
    y2 = ops.gemm(x, w, epilogue=ops.EPI_F32_OUT, scratch=s, pair=True)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert s.error_code() == 0



STREAM_SHAPES = [(48, 3072, 3072), (48, 9216, 3072), (48, 14336, 3072), (48, 3072, 14336),
                 (1, 3072, 3072), (11, 18432, 3072), (64, 2048, 1024), (33, 1536, 640),
                 (16, 4096, 256)]


@pytest.mark.parametrize("m,n,k", STREAM_SHAPES)
def test_gemm_stream_shapes(cuda_device, m, n, k):
    """Token tiles of <= 64 rows: the streaming kernel (full K per CTA, 128
    features each, multi-k-block TMA boxes) where it is planned (N / 128 >= 96,
    K <= 4096: 48 x 14336 x 3072, 11 x 18432 x 3072) and split-K elsewhere:
    raw accumulators against F32, re-tiled weights equal to row-major bit for
    bit, a gated residual written in place over its input."""
    from wam_b200 import ops

    x, w, b = make(m, n, k, seed=m + n + k)
    tw = ops.TiledWeight(w)
    ref = x.float() @ w.float().T
    y_row = ops.gemm(x, w, ops.EPI_F32_OUT)
    y_tiled = ops.gemm(x, tw, ops.EPI_F32_OUT)
    torch.cuda.synchronize()
    # one F32 accumulator per output over the whole K (no split partials): the
    # rounding error grows like sqrt(K)
    assert rel_l2(y_tiled, ref) < 1e-5 * max(1.0, (k / 3072) ** 0.5)
    assert torch.equal(y_row, y_tiled)
    gate = torch.randn(n, device="cuda")
    h = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    expect = bf(h.float() + bf(bf(ref) + b.float()) * gate)
    ops.gemm(x, tw, ops.EPI_GATED_RES, bias=b, gate=gate, residual=h, out=h)
    torch.cuda.synchronize()
    assert rel_l2(h.float(), expect) < 1e-2
