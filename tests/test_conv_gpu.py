"""The implicit-GEMM tcgen05 convolution (csrc/conv.cu) against torch F32
conv2d of the same BF16 operands, with the reference's rounding points
(conv -> BF16, + bias -> BF16, + shortcut -> BF16): 3x3 stride 1 padding 1,
3x3 stride 2 after a one-pixel end pad (the VAE downsampler), 1x1; channel
counts of the Wan VAE encoder (12 -> 16 padded, 96, 160, 320, 640) and
ragged pixel tiles."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def bf(x):
    return x.to(torch.bfloat16).float()


def reference(x, w, b, mode, residual=None):
    xc = x.float().permute(2, 0, 1)[None]
    if mode == 1:
        xc = F.pad(xc, (0, 1, 0, 1))
        y = F.conv2d(xc, w.float(), stride=2)
    else:
        y = F.conv2d(xc, w.float(), padding=1 if mode == 0 else 0)
    y = bf(bf(y[0].permute(1, 2, 0)) + b.float())
    if residual is not None:
        y = bf(y + residual.float())
    return y


@pytest.mark.parametrize("h,w,cin,cout,mode", [
    (24, 32, 160, 160, 0),    # down block 0 resnet conv
    (16, 48, 320, 640, 0),    # down block 2 resnet conv1 (Cout over 3 N tiles)
    (8, 16, 64, 160, 0),      # conv_in on the 12-channel patchified input padded to 64
    (13, 20, 64, 96, 0),      # ragged pixel tiles, conv_out-sized Cout
    (6, 6, 640, 96, 0),       # 36 pixels (one partial tile)
    (32, 48, 160, 160, 1),    # downsampler of block 0
    (16, 16, 320, 320, 1),    # downsampler of block 1
    (10, 34, 640, 640, 1),    # odd output width (17): ragged tile at the right edge
    (24, 32, 160, 320, 2),    # conv_shortcut 160 -> 320
    (48, 64, 96, 96, 2),      # quant_conv
])
def test_conv_vs_torch(cuda_device, h, w, cin, cout, mode):
    from wam_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(h * 1000 + w * 10 + cin + mode)
    k = 1 if mode == 2 else 3
    x = torch.randn(h, w, cin, generator=g).to(torch.bfloat16).cuda()
    wt = (torch.randn(cout, cin, k, k, generator=g) * (1.0 / (cin * k * k) ** 0.5)).to(
        torch.bfloat16).cuda()
    b = (torch.randn(cout, generator=g) * 0.1).to(torch.bfloat16).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.conv2d(x, ops.ConvWeight(wt), mode, bias=b, error=err)
    ref = reference(x, wt, b, mode)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert y.shape == ref.shape
    d = (y.float() - ref)
    # F32 accumulation order differs from torch's: allow one BF16 rounding flip.
    assert (d.abs() <= ref.abs() * 2 ** -7 + 1e-3).float().mean() > 0.999
    assert (d.norm() / ref.norm()).item() < 4e-3


@pytest.mark.parametrize("mode", [0, 1])
def test_conv_residual_epilogue(cuda_device, mode):
    from wam_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(77 + mode)
    h, w, c = 16, 32, 160
    x = torch.randn(h, w, c, generator=g).to(torch.bfloat16).cuda()
    wt = (torch.randn(c, c, 3, 3, generator=g) * (1.0 / (9 * c) ** 0.5)).to(torch.bfloat16).cuda()
    b = (torch.randn(c, generator=g) * 0.1).to(torch.bfloat16).cuda()
    oh, ow = (h // 2, w // 2) if mode == 1 else (h, w)
    r = torch.randn(oh, ow, c, generator=g).to(torch.bfloat16).cuda()
    y = ops.conv2d(x, ops.ConvWeight(wt), mode, bias=b, residual=r)
    ref = reference(x, wt, b, mode, residual=r)
    torch.cuda.synchronize()
    assert ((y.float() - ref).norm() / ref.norm()).item() < 4e-3


def test_conv_rejects_bad_shapes(cuda_device):
    from wam_b200 import ops

    x = torch.zeros(8, 8, 12, dtype=torch.bfloat16, device="cuda")  # narrower than a channel block
    wt = ops.ConvWeight(torch.zeros(16, 12, 3, 3, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError, match="at least 64"):
        ops.conv2d(x, wt, 0)
    x = torch.zeros(8, 8, 68, dtype=torch.bfloat16, device="cuda")  # 136-byte rows
    wt = ops.ConvWeight(torch.zeros(16, 68, 3, 3, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.conv2d(x, wt, 0)
    x = torch.zeros(7, 8, 64, dtype=torch.bfloat16, device="cuda")
    wt = ops.ConvWeight(torch.zeros(16, 64, 3, 3, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError, match="even input"):
        ops.conv2d(x, wt, 1)
