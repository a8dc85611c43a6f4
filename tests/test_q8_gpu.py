"""Q8_0 weights on the device: quantiser bit-exact against gguf-py, tile
layout, and the GEMM that converts Q8_0 tiles to BF16 in shared memory
(compared with an F32 matmul of the dequantised weights rounded to BF16, the
engine's documented Q8_0 semantics)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")
from gguf import quants  # noqa: E402


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def dequant_bf16(blocks, n, k):
    d = blocks[:, :2].contiguous().view(torch.float16).float()
    q = blocks[:, 2:].contiguous().view(torch.int8).float()
    return (q * d).reshape(n, k).to(torch.bfloat16)


@pytest.mark.parametrize("n,k", [(256, 64), (512, 3072), (3072, 256)])
def test_q8_quantize_matches_gguf(cuda_device, n, k):
    from wam_b200 import ops

    g = torch.Generator().manual_seed(n + k)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    w[0, :32] = torch.linspace(-1, 1, 32) * (127 / 64)  # exact .5 ties after scaling
    w[1, :32] = 0
    got = ops.q8_quantize(w.cuda()).cpu().numpy()
    ref = quants.quantize(w.float().numpy(), gguf.GGMLQuantizationType.Q8_0).reshape(-1, 34)
    assert np.array_equal(got, ref)


def test_q8_retile_layout(cuda_device):
    from wam_b200 import ops

    n, k = 512, 128
    w = (torch.randn(n, k) * 0.02).to(torch.bfloat16).cuda()
    qw = ops.Q8Weight(w)
    blocks = qw.blocks.cpu().view(n, k // 32, 34)
    tiles = qw.data.cpu().view(n // 256, k // 64, ops.Q8_TILE_BYTES)
    for nt in range(n // 256):
        for kb in range(k // 64):
            t = tiles[nt, kb]
            q = t[:16384].view(256, 64)
            d = t[16384:].view(256, 2, 2)
            for r in (0, 7, 128, 255):
                for h in range(2):
                    blk = blocks[nt * 256 + r, kb * 2 + h]
                    assert torch.equal(q[r, h * 32:(h + 1) * 32], blk[2:])
                    assert torch.equal(d[r, h], blk[:2])


@pytest.mark.parametrize("m,n,k", [(48, 3072, 3072), (1, 512, 256), (768, 1024, 512),
                                   (200, 512, 640), (48, 3072, 14336)])
@pytest.mark.parametrize("mode", ["cluster", "workspace"])
def test_q8_gemm(cuda_device, m, n, k, mode):
    from wam_b200 import ops

    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    qw = ops.Q8Weight(w)
    wd = dequant_bf16(qw.blocks, n, k)
    s = ops.Scratch() if mode == "workspace" else None
    y = ops.gemm(x, qw, ops.EPI_F32_OUT, scratch=s)
    ref = x.float() @ wd.float().T
    torch.cuda.synchronize()
    assert rel_l2(y, ref) < 1e-5
    # identical to the BF16 GEMM on the dequantised weights, bit for bit
    y2 = ops.gemm(x, wd, ops.EPI_F32_OUT, scratch=s)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    yb = ops.gemm(x, qw, ops.EPI_BIAS_GELU, bias=b, scratch=s)
    yb2 = ops.gemm(x, wd, ops.EPI_BIAS_GELU, bias=b, scratch=s)
    torch.cuda.synchronize()
    assert torch.equal(yb, yb2)
