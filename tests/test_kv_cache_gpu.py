"""KV-cache indexing, exactly: the Q/K/V post-processing kernel that writes the
engine's caches (wam_b200_op_qkv_scatter; expert_qkv, src/models/gwp05/engine/
mot.cpp:210-267, and the cache layout of engine/cache.cpp:441-469 in this
engine's head-major form) at config-2 shapes: 24 heads x 128, 768 visual rows
of a 32 x 24 grid with 3-D RoPE written at rows 1..768, the state token at row
0, 48 action rows with 1-D RoPE at rows 769..816, two requests.

* V is a cast, so every cached V element must equal its source bit for bit.
* Q and K go through F32 RMSNorm and RoPE: compared with a numpy F32
  restatement within 1e-2 relative-L2 and 2 BF16 ulps per element, and every
  row must be nearest to the restatement's row of the same index.
* Rows the launch does not own keep their sentinel value.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HEADS, V_ROWS, T_ROWS = 24, 768, 48
P = 1 + V_ROWS
H = HEADS * 128
SENT = 12288.0  # exactly representable in BF16


def rope_ref(x, pos, sections):
    """x: [rows, H] F32 after RMSNorm; pos: [rows, n_sections]; sections: dims."""
    out = x.copy()
    rows = x.shape[0]
    for h in range(HEADS):
        d0 = h * 128
        for k, nd in enumerate(sections):
            ts = np.float32(10000.0) ** np.float32(-2.0 / nd)
            inv = np.array([np.float32(ts) ** np.float32(i) for i in range(nd // 2)], np.float32)
            theta = (pos[:, k:k + 1].astype(np.float32) * inv[None, :]).astype(np.float64)
            c, s = np.cos(theta), np.sin(theta)
            x0 = out[:, d0 + 0:d0 + nd:2].astype(np.float64)
            x1 = out[:, d0 + 1:d0 + nd:2].astype(np.float64)
            out[:, d0 + 0:d0 + nd:2] = (x0 * c - x1 * s).astype(np.float32)
            out[:, d0 + 1:d0 + nd:2] = (x0 * s + x1 * c).astype(np.float32)
            d0 += nd
    assert out.shape[0] == rows
    return out


def rms_ref(x, w, eps=1e-6):
    x = x.astype(np.float32)
    inv = 1.0 / np.sqrt((x * x).mean(axis=1, keepdims=True) + np.float32(eps))
    return (x * inv * w[None, :]).astype(np.float32)


def to_heads(x, rows):
    return x.reshape(-1, rows, HEADS, 128).transpose(0, 2, 1, 3)


def close_and_in_place(got, want, label):
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    rel = np.linalg.norm(g - w) / np.linalg.norm(w)
    assert rel < 1e-2, f"{label}: rel-L2 {rel:.3e}"
    assert (np.abs(g - w) <= 2 ** -6 * np.abs(w) + 1e-3).all(), f"{label}: element off by > 2 ulps"
    for b in range(g.shape[0]):
        for h in range(g.shape[1]):
            gg, ww = g[b, h], w[b, h]
            d = (gg * gg).sum(1)[:, None] + (ww * ww).sum(1)[None, :] - 2.0 * gg @ ww.T
            assert (np.argmin(d, axis=1) == np.arange(gg.shape[0])).all(), (
                f"{label}: rows of request {b} head {h} out of place")


def _setup(rows_per_seq, batch=2, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    src = torch.randn(batch * rows_per_seq, 3 * H, generator=g).to(torch.bfloat16)
    qn = (1 + 0.02 * torch.randn(H, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.02 * torch.randn(H, generator=g)).to(torch.bfloat16)
    kc = torch.full((batch, HEADS, P + T_ROWS, 128), SENT, dtype=torch.bfloat16)
    vc = kc.clone()
    return src, qn, kn, kc, vc


def test_visual_rows_exact_placement(cuda_device):
    from wam_b200 import ops

    src, qn, kn, kc, vc = _setup(V_ROWS)
    qo = torch.full((2, HEADS, P, 128), SENT, dtype=torch.bfloat16)
    pos = np.array([(0, y, x) for y in range(32) for x in range(24)], np.int32)
    src_d, kc_d, vc_d, qo_d = src.cuda(), kc.cuda(), vc.cuda(), qo.cuda()
    ops.qkv_scatter(src_d, HEADS, V_ROWS, q_out=qo_d, k_out=kc_d, v_out=vc_d, q_norm=qn.cuda(),
                    k_norm=kn.cuda(), rope_mode=2, pos_thw=torch.from_numpy(pos).cuda(),
                    q_row_offset=1, kv_row_offset=1, cols=(0, H, 2 * H))
    torch.cuda.synchronize()
    k_got = kc_d.float().cpu().numpy()
    v_got = vc_d.float().cpu().numpy()
    q_got = qo_d.float().cpu().numpy()
    s = src.float().numpy()
    # V: exact, at rows 1..768
    assert np.array_equal(v_got[:, :, 1:P], to_heads(s[:, 2 * H:], V_ROWS))
    for cache in (k_got, v_got):
        assert (cache[:, :, 0] == SENT).all() and (cache[:, :, P:] == SENT).all()
    assert (q_got[:, :, 0] == SENT).all()
    posr = np.tile(pos, (2, 1))
    for part, col, w, got in (("k", H, kn, k_got), ("q", 0, qn, q_got)):
        ref = rope_ref(rms_ref(s[:, col:col + H], w.float().numpy()), posr, (44, 42, 42))
        ref_b = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
        close_and_in_place(got[:, :, 1:P], to_heads(ref_b, V_ROWS), f"visual {part}")


@pytest.mark.parametrize("rows,offset,pos_base", [(T_ROWS, P, 1), (1, 0, 0)])
def test_action_and_state_rows_exact_placement(cuda_device, rows, offset, pos_base):
    """Action rows (positions 1..48, rows P..P+47) and the state row (position 0, row 0)."""
    from wam_b200 import ops

    src, qn, kn, kc, vc = _setup(rows, seed=rows)
    qo = torch.full((2, HEADS, rows, 128), SENT, dtype=torch.bfloat16).cuda()
    kd, vd = kc.cuda(), vc.cuda()
    ops.qkv_scatter(src.cuda(), HEADS, rows, q_out=qo, k_out=kd, v_out=vd, q_norm=qn.cuda(),
                    k_norm=kn.cuda(), rope_mode=1, pos_base=pos_base, kv_row_offset=offset,
                    cols=(0, H, 2 * H))
    torch.cuda.synchronize()
    s = src.float().numpy()
    k_got, v_got = kd.float().cpu().numpy(), vd.float().cpu().numpy()
    assert np.array_equal(v_got[:, :, offset:offset + rows], to_heads(s[:, 2 * H:], rows))
    mask = np.ones(P + T_ROWS, bool)
    mask[offset:offset + rows] = False
    assert (k_got[:, :, mask] == SENT).all() and (v_got[:, :, mask] == SENT).all()
    posr = np.tile(np.arange(pos_base, pos_base + rows, dtype=np.int32)[:, None], (2, 1))
    for part, col, w, got in (("k", H, kn, k_got[:, :, offset:offset + rows]),
                              ("q", 0, qn, qo.float().cpu().numpy())):
        ref = rope_ref(rms_ref(s[:, col:col + H], w.float().numpy()), posr, (128,))
        ref_b = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
        close_and_in_place(got, to_heads(ref_b, rows), f"rows@{offset} {part}")
