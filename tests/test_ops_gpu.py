"""Attention, LayerNorm and synthetic-weight kernels against CPU/torch restatements.

Attention and LayerNorm are floating-point kernels: their reference is a torch
F32 computation on the same BF16 inputs (tolerance: 1e-2 relative-L2 for
attention, per the attention-microbench bar; LayerNorm outputs within one BF16
ulp on >99.9% of elements). The synthetic generator is integer/byte work:
bit-exact against the numpy generator in oracle/synth.py.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def torch_attention(q, k, v, scale):
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * scale
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhqk,bhkd->bhqd", p, v.float())
    B, H, Lq, D = o.shape
    return o.permute(0, 2, 1, 3).reshape(B * Lq, H * D)


@pytest.mark.parametrize("B,heads,lq,lk", [
    (1, 24, 48, 817),      # denoise self-attention at config 2 (P + T keys)
    (1, 24, 48, 512),      # denoise cross-attention over the prompt
    (1, 4, 769, 769),      # prefix joint self-attention (heads reduced)
    (2, 3, 1, 64),         # state token cross-attention
    (3, 2, 100, 1280),     # ragged queries, microbench cache length
    (1, 2, 816, 4096),     # microbench: 48 + 768 queries over a 4096 cache
    (8, 24, 816, 1280),    # config 3: batch 8 over the 1280-key cache, 24 heads
    (1, 24, 816, 16384),   # config 3: the 16384-key cache, 24 heads
    (1, 24, 816, 1280),    # config 3 batch 1: 168 CTAs (1.14 waves)
    (1, 24, 769, 769),     # prefix joint attention at config-2 widths, ragged last key tile
])
def test_attention_vs_torch(cuda_device, B, heads, lq, lk):
    _attention_case(B, heads, lq, lk, 1.0)


@pytest.mark.parametrize("B,heads,lq,lk,qs", [
    (2, 24, 48, 817, 1.0),    # batch 2: 4 key splits of 2 tiles (online softmax across tiles)
    (8, 24, 48, 817, 1.0),    # batch 8: one CTA per (sequence, head), 7 key tiles
    (1, 24, 1, 512, 1.0),     # prefix state token over the prompt keys
    (1, 2, 64, 3000, 4.0),    # 64 query rows, 24 tiles per CTA, wide scores (O rescaled)
    (3, 5, 33, 250, 8.0),     # ragged rows / keys, very wide scores
    (1, 2, 64, 896, 4.0),     # 64 queries, seven full key tiles (every TMEM column)
    (2, 4, 17, 1, 1.0),       # a single key
    (1, 3, 40, 129, 1.0),     # two key tiles, the second with one key; 40 queries (N = 48)
])
def test_decode_attention_vs_torch(cuda_device, B, heads, lq, lk, qs):
    """The decode attention (<= 64 queries per head: the tcgen05 kernel of
    attention_dec_tc.cu, one CTA or a cluster of 2 / 4 key-split CTAs per
    (sequence, head); the mma.sync kernel beyond 896 keys) against torch F32,
    including ragged key tiles and wide score ranges."""
    _attention_case(B, heads, lq, lk, qs)


_DECODE_CASES = r"""
import sys
sys.path.insert(0, "wam.cpp_b200")
import torch
from wam_b200 import ops

def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))

cases = [(1, 24, 48, 817, 1.0), (1, 24, 48, 512, 1.0), (2, 3, 1, 64, 1.0), (1, 24, 1, 512, 1.0),
         (3, 5, 33, 250, 8.0), (1, 2, 64, 896, 4.0), (2, 4, 17, 1, 1.0), (1, 3, 40, 129, 1.0),
         (2, 24, 48, 817, 1.0), (1, 24, 769, 769, 1.0)]
worst = 0.0
for B, H, lq, lk, qs in cases:
    g = torch.Generator().manual_seed(lq * 31 + lk)
    q = (torch.randn(B, H, lq, 128, generator=g) * qs).to(torch.bfloat16).cuda()
    k = torch.randn(B, H, lk, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, H, lk, 128, generator=g).to(torch.bfloat16).cuda()
    y = ops.attention(q, k, v)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) / 128 ** 0.5
    o = torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, dim=-1), v.float())
    ref = o.permute(0, 2, 1, 3).reshape(B * lq, H * 128)
    torch.cuda.synchronize()
    err = rel_l2(y.float(), ref)
    if not torch.isfinite(y.float()).all() or err >= 1e-2:
        raise SystemExit(f"case {(B, H, lq, lk, qs)}: rel-L2 {err}")
    worst = max(worst, err)
print("worst rel-L2", worst)
"""


def test_decode_attention_mma_sync(cuda_device):
    """The mma.sync decode kernel (attention.cu: 64-query blocks, keys split
    over up to 8 CTAs merged through L2 or distributed shared memory), which
    the tcgen05 kernel replaces for <= 896 keys, on the same shapes and on the
    one-row ragged tail of a 769-query launch: WAM_B200_ATTN_DEC_TC=0 in a
    child process."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    env = dict(os.environ, WAM_B200_ATTN_DEC_TC="0")
    r = subprocess.run([sys.executable, "-c", _DECODE_CASES], env=env, capture_output=True, text=True,
                       cwd=str(Path(__file__).resolve().parent.parent), timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr


def _attention_case(B, heads, lq, lk, qs):
    from wam_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(lq * 31 + lk)
    q = (torch.randn(B, heads, lq, 128, generator=g) * qs).to(torch.bfloat16).cuda()
    k = torch.randn(B, heads, lk, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, heads, lk, 128, generator=g).to(torch.bfloat16).cuda()
    y = ops.attention(q, k, v)
    ref = torch_attention(q, k, v, 1.0 / 128 ** 0.5)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    assert rel_l2(y.float(), ref) < 1e-2


@pytest.mark.parametrize("rows,cols", [(48, 3072), (769, 3072), (5, 256), (3, 4096), (3072, 3072),
                                       (1500, 4096)])
@pytest.mark.parametrize("affine", [False, True])
def test_layernorm_vs_torch(cuda_device, rows, cols, affine):
    from wam_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) * 3 + 0.5).to(torch.bfloat16).cuda()
    if affine:
        a = (1 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16).cuda()
        b = (0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16).cuda()
    else:
        a = (0.1 * torch.randn(cols, generator=g)).float().cuda()
        b = (0.1 * torch.randn(cols, generator=g)).float().cuda()
    y = ops.layernorm(x, a, b, eps=1e-6, affine=affine)
    xf = x.float()
    mu = xf.mean(dim=1, keepdim=True)
    var = ((xf - mu) ** 2).mean(dim=1, keepdim=True)
    n = (xf - mu) / torch.sqrt(var + 1e-6)
    ref = n * a.float() + b.float() if affine else n * (1 + a) + b
    ref = ref.to(torch.bfloat16).float()
    torch.cuda.synchronize()
    yf = y.float()
    ulp = torch.clamp(ref.abs(), min=1e-3) * 2.0 ** -7
    assert ((yf - ref).abs() > 1.01 * ulp).float().mean().item() < 1e-3
    assert rel_l2(yf, ref) < 5e-3


@pytest.mark.parametrize("affine", [False, True])
def test_layernorm_many_rows_bit_identical(cuda_device, affine):
    """>= 1024 rows take the streaming LayerNorm kernel; the same rows in
    launches of 512 take the latency kernel. Same arithmetic: same bits."""
    from wam_b200 import ops

    rows, cols = 2048, 3072
    g = torch.Generator(device="cpu").manual_seed(77)
    x = (torch.randn(rows, cols, generator=g) * 2 - 0.3).to(torch.bfloat16).cuda()
    if affine:
        a = (1 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16).cuda()
        b = (0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16).cuda()
    else:
        a = (0.1 * torch.randn(cols, generator=g)).float().cuda()
        b = (0.1 * torch.randn(cols, generator=g)).float().cuda()
    y = ops.layernorm(x, a, b, eps=1e-6, affine=affine)
    parts = [ops.layernorm(x[i:i + 512].contiguous(), a, b, eps=1e-6, affine=affine)
             for i in range(0, rows, 512)]
    torch.cuda.synchronize()
    assert torch.equal(y, torch.cat(parts))


@pytest.mark.parametrize("name,n,scale,center", [
    ("gwp.blk.0.a.sa.qkv.weight", 1 << 20, 0.02, 0.0),
    ("gwp.blk.3.v.sa.qn.weight", 3072, 0.02, 1.0),
    ("gwp.patch.bias", 1000, 0.02, 0.0),
])
def test_synthetic_weights_bit_exact(cuda_device, name, n, scale, center):
    from oracle import synth
    from wam_b200 import ops

    dev = ops.synth(n, 1234, name, scale, center).view(torch.int16).cpu().numpy().view(np.uint16)
    host = synth.synth_bits(1234, name, n, scale, center)
    assert np.array_equal(dev, host)
