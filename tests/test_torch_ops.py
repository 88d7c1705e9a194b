"""torch.ops.b200msat: the op-level counterparts of the reference's ds:: / ss:: custom ops.

CPU: every op is registered with a fake implementation that gives the reference op's output
shapes.  GPU: each op against a plain PyTorch fp32 restatement of the reference op's arithmetic
on the same inputs (bf16 rounding where the reference rounds)."""

import pytest
import torch
import torch.nn.functional as F

import rldx_b200.torch_ops  # noqa: F401  (registers torch.ops.b200msat)

BF = torch.bfloat16
OPS = ["ds_fused_attention_2way", "ds_fused_attention_3way", "ss_fused_attention_2way",
       "ss_fused_attention_3way", "ds_grouped_res_ln", "ds_grouped_swiglu", "ds_vl_epilogue_ln",
       "ss_fused_epilogue_ln", "ss_fused_mlp_swiglu", "linear", "joint_attention", "layernorm",
       "qk_rmsnorm_rope", "swiglu"]


def test_ops_registered():
    for name in OPS:
        assert hasattr(torch.ops.b200msat, name), name


def test_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        H, n_sa, n_vl, n_p = 4, 18, 40, 32
        sa, vl, p = (torch.empty(n, 3 * H * 64, dtype=BF) for n in (n_sa, n_vl, n_p))
        w = torch.empty(64, dtype=BF)
        c = torch.empty(n_sa, 32)
        out = torch.ops.b200msat.ds_fused_attention_3way(sa, vl, p, w, w, w, w, w, w, c, c, c, c, n_sa, n_vl, n_p)
        assert tuple(out.shape) == (1, n_sa + n_vl + n_p, H * 64)
        out = torch.ops.b200msat.ss_fused_attention_2way(vl, w, w, c, c, n_sa)
        assert tuple(out.shape) == (1, n_vl, H * 64)
        a, b = torch.ops.b200msat.ds_grouped_swiglu(torch.empty(n_sa, 512, dtype=BF), torch.empty(512, dtype=BF),
                                                    torch.empty(n_vl, 768, dtype=BF), torch.empty(768, dtype=BF),
                                                    n_sa, n_vl, 256, 384)
        assert tuple(a.shape) == (n_sa, 256) and tuple(b.shape) == (n_vl, 384)
        new, ln = torch.ops.b200msat.ss_fused_epilogue_ln(torch.empty(1, 7, 256, dtype=BF), torch.empty(1, 7, 256, dtype=BF))
        assert tuple(new.shape) == tuple(ln.shape) == (1, 7, 256)


# ------------------------------------------------------------------------------------------------
# GPU parity
# ------------------------------------------------------------------------------------------------
def _rms(x, w, eps=1e-6):
    xf = x.float()
    return (w.float() * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps))).to(BF)


def _rope(x, cos, sin):
    """Interleaved-pair rotation in fp32, one rounding (ops.py:48-67)."""
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    a, b = xf[..., 0], xf[..., 1]
    return torch.stack([a * cos - b * sin, a * sin + b * cos], dim=-1).flatten(-2).to(BF)


def _ref_attention(segments, H):
    """segments: (qkv [n, 3*H*64], qn, kn, cos or None, sin, rope_from)."""
    qs, ks, vs = [], [], []
    for qkv, qn, kn, cos, sin, rf in segments:
        n = qkv.shape[0]
        q, k, v = (t.reshape(n, H, 64).transpose(0, 1) for t in qkv.chunk(3, dim=-1))
        q, k = _rms(q, qn), _rms(k, kn)
        if cos is not None:
            c, s = cos[None], sin[None]  # [1, n - rf, 32]
            q = torch.cat([q[:, :rf], _rope(q[:, rf:], c, s)], dim=1)
            k = torch.cat([k[:, :rf], _rope(k[:, rf:], c, s)], dim=1)
        qs.append(q), ks.append(k), vs.append(v)
    q, k, v = torch.cat(qs, 1), torch.cat(ks, 1), torch.cat(vs, 1)
    o = torch.softmax((q.float() @ k.float().transpose(-1, -2)) / 8.0, -1) @ v.float()
    return o.transpose(0, 1).reshape(1, -1, H * 64)


def _tables(n, g, dev):
    ang = torch.rand(n, 32, device=dev, generator=g) * 6.0
    return ang.cos(), ang.sin()


@pytest.mark.gpu
@pytest.mark.parametrize("H,n_vl,n_sa,n_p", [(4, 40, 18, 32), (24, 512, 18, 32)])
def test_ds_fused_attention_3way(cuda, H, n_vl, n_sa, n_p):
    g = torch.Generator(device=cuda).manual_seed(H + n_vl)
    mk = lambda n: torch.randn(n, 3 * H * 64, device=cuda, generator=g).to(BF)  # noqa: E731
    nw = lambda: (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)  # noqa: E731
    sa, vl, p = mk(n_sa), mk(n_vl), mk(n_p)
    w = [nw() for _ in range(6)]
    sc, ss = _tables(n_sa, g, cuda)
    pc, ps = _tables(n_p, g, cuda)
    out = torch.ops.b200msat.ds_fused_attention_3way(sa, vl, p, w[0], w[1], w[2], w[3], w[4], w[5],
                                                     sc, ss, pc, ps, n_sa, n_vl, n_p)
    ref = _ref_attention([(vl, w[2], w[3], None, None, 0), (sa, w[0], w[1], sc, ss, 0),
                          (p, w[4], w[5], pc, ps, 0)], H)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.gpu
def test_ds_fused_attention_2way(cuda):
    H, n_vl, n_sa = 4, 64, 17
    g = torch.Generator(device=cuda).manual_seed(2)
    sa = torch.randn(n_sa, 3 * H * 64, device=cuda, generator=g).to(BF)
    vl = torch.randn(n_vl, 3 * H * 64, device=cuda, generator=g).to(BF)
    w = [(1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF) for _ in range(4)]
    c, s = _tables(n_sa, g, cuda)
    out = torch.ops.b200msat.ds_fused_attention_2way(sa, vl, w[0], w[1], w[2], w[3], c, s, n_sa, n_vl)
    ref = _ref_attention([(vl, w[2], w[3], None, None, 0), (sa, w[0], w[1], c, s, 0)], H)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.gpu
def test_ss_fused_attention_2way_and_3way(cuda):
    H, n_x, n_sa, n_p = 4, 82, 17, 32
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(n_x, 3 * H * 64, device=cuda, generator=g).to(BF)
    p = torch.randn(n_p, 3 * H * 64, device=cuda, generator=g).to(BF)
    w = [(1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF) for _ in range(4)]
    sc, ss = _tables(n_sa, g, cuda)
    pc, ps = _tables(n_p, g, cuda)
    out2 = torch.ops.b200msat.ss_fused_attention_2way(x, w[0], w[1], sc, ss, n_sa)
    ref2 = _ref_attention([(x, w[0], w[1], sc, ss, n_x - n_sa)], H)
    out3 = torch.ops.b200msat.ss_fused_attention_3way(x, p, w[0], w[1], w[2], w[3], sc, ss, pc, ps, n_x, n_sa, n_p)
    ref3 = _ref_attention([(x, w[0], w[1], sc, ss, n_x - n_sa), (p, w[2], w[3], pc, ps, 0)], H)
    torch.cuda.synchronize()
    assert (out2.float() - ref2).abs().max().item() < 2e-2
    assert (out3.float() - ref3).abs().max().item() < 2e-2


@pytest.mark.gpu
def test_epilogue_ops(cuda):
    g = torch.Generator(device=cuda).manual_seed(4)
    r = lambda *s: torch.randn(*s, device=cuda, generator=g).to(BF)  # noqa: E731
    m_sa, m_vl, d_sa, d_vl = 18, 64, 256, 512
    # ds::grouped_res_ln: LN(res + proj + bias) summed in fp32
    sa_res, sa_proj, sa_b = r(1, m_sa, d_sa), r(m_sa, d_sa), r(d_sa)
    vl_res, vl_proj, vl_b = r(1, m_vl, d_vl), r(m_vl, d_vl), r(d_vl)
    a, b = torch.ops.b200msat.ds_grouped_res_ln(sa_res, sa_b, sa_proj, vl_res, vl_b, vl_proj, m_sa, m_vl, d_sa, d_vl)
    ra = F.layer_norm(sa_res[0].float() + sa_proj.float() + sa_b.float(), (d_sa,), eps=1e-6).to(BF)
    rb = F.layer_norm(vl_res[0].float() + vl_proj.float() + vl_b.float(), (d_vl,), eps=1e-6).to(BF)
    # ds::vl_epilogue_ln: bf16 after each add, then LN
    pb, wb, w3 = r(d_vl), r(d_vl), r(m_vl, d_vl)
    new, ln = torch.ops.b200msat.ds_vl_epilogue_ln(vl_res, pb, wb, w3, m_vl, d_vl)
    rnew = ((vl_res[0] + pb) + wb) + w3
    rln = F.layer_norm(rnew.float(), (d_vl,), eps=1e-6).to(BF)
    # ss::fused_epilogue_ln
    hid, res = r(1, m_vl, d_sa), r(1, m_vl, d_sa)
    new2, ln2 = torch.ops.b200msat.ss_fused_epilogue_ln(hid, res)
    rnew2 = hid + res
    rln2 = F.layer_norm(rnew2.float(), (d_sa,), eps=1e-6).to(BF)
    # ds::grouped_swiglu: fp32 bias + silu * up, one rounding
    w12s, bs, w12v, bv = r(m_sa, 2 * 128), r(2 * 128), r(m_vl, 2 * 192), r(2 * 192)
    s_out, v_out = torch.ops.b200msat.ds_grouped_swiglu(w12s, bs, w12v, bv, m_sa, m_vl, 128, 192)

    def sw(x, bias, h):
        gt, up = x.float()[:, :h] + bias.float()[:h], x.float()[:, h:] + bias.float()[h:]
        return (F.silu(gt) * up).to(BF)

    torch.cuda.synchronize()
    for got, exp in ((a[0], ra), (b[0], rb), (ln[0], rln), (ln2, rln2), (s_out, sw(w12s, bs, 128)),
                     (v_out, sw(w12v, bv, 192))):
        d = (got.float() - exp.float()).abs()
        assert d.max().item() <= 2 ** -6 * max(1.0, exp.float().abs().max().item()), d.max().item()
        assert (d > 0).float().mean().item() < 0.01
    assert torch.equal(new[0], rnew) and torch.equal(new2, rnew2)


@pytest.mark.gpu
def test_ss_fused_mlp_swiglu(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(82, 256, device=cuda, generator=g).to(BF)
    w = (0.05 * torch.randn(2 * 384, 256, device=cuda, generator=g)).to(BF)
    b = (0.1 * torch.randn(2 * 384, device=cuda, generator=g)).to(BF)
    out = torch.ops.b200msat.ss_fused_mlp_swiglu(x, w, b)
    acc = x.float() @ w.float().t() + b.float()
    ref = F.silu(acc[:, :384]) * acc[:, 384:]
    torch.cuda.synchronize()
    # the projection is rounded to bf16 before the bias (the reference keeps it in fp32): a
    # couple of bf16 ulps of the output's magnitude
    assert (out.float() - ref).abs().max().item() <= 2 ** -6 * max(1.0, ref.abs().max().item())
