"""Memory-bound row kernels vs plain PyTorch references (same bf16 rounding points)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200 import ops  # noqa: E402

BF = torch.bfloat16


@pytest.mark.parametrize("rows,D", [(1, 64), (18, 1536), (562, 1536), (77, 4096), (5, 1024)])
def test_layernorm(cuda, rows, D):
    g = torch.Generator(device=cuda).manual_seed(rows + D)
    x = (torch.randn(rows, D, device=cuda, generator=g) * 3 + 1).to(BF)
    out = ops.layernorm(x)
    ref = F.layer_norm(x.float(), (D,), eps=1e-6).to(BF)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max() <= 2 ** -6


def test_layernorm_modulate(cuda):
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(18, 1536, device=cuda, generator=g).to(BF)
    sc1p = (1 + 0.2 * torch.randn(1536, device=cuda, generator=g)).to(BF)
    sh = (0.2 * torch.randn(1536, device=cuda, generator=g)).to(BF)
    out = ops.layernorm(x, scale1p=sc1p, shift=sh)
    ln = F.layer_norm(x.float(), (1536,), eps=1e-6).to(BF)
    ref = (ln * sc1p + sh)  # bf16 tensor ops: two roundings, as msat.py:780
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max() <= 2 ** -5


def qwen3_ref(x, w, cos, sin, pos, eps=1e-6):
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(BF)
    y = w * xn
    c, s = cos[pos][:, None], sin[pos][:, None]
    rot = torch.cat([-y[..., 64:], y[..., :64]], dim=-1)
    return y * c + rot * s


@pytest.mark.parametrize("T,H", [(1, 1), (37, 16), (4096, 16)])
def test_qk_rmsnorm_rope_qwen3(cuda, T, H):
    g = torch.Generator(device=cuda).manual_seed(T)
    x = torch.randn(T, H, 128, device=cuda, generator=g).to(BF)
    w = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).to(BF)
    pos = (torch.arange(T, device=cuda) % 4096).to(torch.int32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=cuda).float() / 128))
    freqs = torch.outer(torch.arange(4096, device=cuda).float(), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    cos, sin = emb.cos().to(BF), emb.sin().to(BF)
    out = ops.qk_rmsnorm_rope(x, w, pos, cos, sin)
    ref = qwen3_ref(x, w, cos, sin, pos.long())
    torch.cuda.synchronize()
    d = (out.float() - ref.float()).abs()
    assert d.max() <= 2 ** -5 * ref.float().abs().max()
    assert (d > 0).float().mean() < 0.01


@pytest.mark.parametrize("rows,H", [(1, 8), (65536 // 64, 8960), (300, 4096)])
def test_swiglu(cuda, rows, H):
    g = torch.Generator(device=cuda).manual_seed(rows)
    x = torch.randn(rows, 2 * H, device=cuda, generator=g).to(BF)
    gate, up = x[:, :H], x[:, H:]
    out = ops.swiglu(gate, up)
    ref = F.silu(gate) * up
    torch.cuda.synchronize()
    d = (out.float() - ref.float()).abs()
    assert d.max() <= 2 ** -7 * ref.float().abs().max() + 1e-6
    assert (d > 0).float().mean() < 0.01
