"""tcgen05 grouped GEMM vs a plain PyTorch fp32 reference of the same op (same bf16 rounding
points), across tile widths, ragged M/N/K, every epilogue and the category-weight path."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200 import _lib, ops  # noqa: E402

BF = torch.bfloat16


def r(x):
    return x.to(BF).float()


def ref_finish(acc, b, bias_mode, act):
    if bias_mode == _lib.BIAS_FUSED:
        y = r(acc + b.float())
    elif bias_mode == _lib.BIAS_POST_ROUND:
        y = r(r(acc) + b.float())
    else:
        y = r(acc)
    if act == _lib.ACT_RELU:
        y = torch.relu(y)
    elif act == _lib.ACT_SILU:
        y = r(F.silu(y))
    elif act == _lib.ACT_SWISH:
        y = r(y * r(torch.sigmoid(y)))
    return y


def close(out, ref, tol=2e-2, rel_tol=1e-2):
    """Max error within tol of the output's magnitude, and the relative RMS error within rel_tol:
    the reference applies the same bf16 roundings, so a correct kernel differs from it only where
    fp32 sums in another order round the other way (relative RMS ~1e-3)."""
    out = out.float()
    scale = ref.abs().max().clamp_min(1e-3)
    err = (out - ref).abs().max()
    assert err <= tol * scale, f"max err {err.item():.4g} vs scale {scale.item():.4g}"
    rel = ((out - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert rel <= rel_tol, f"relative RMS error {rel:.4g}"
    # bf16 rounding of an fp32 sum in another order: almost every element is exact or 1 ulp off
    bad = ((out - ref).abs() > 2 ** -7 * ref.abs() + 1e-3 * scale).float().mean()
    assert bad < 0.01, f"{bad.item():.3%} elements beyond 1 ulp"


SHAPES = [(1, 64, 64), (18, 4608, 1536), (32, 1536, 4096), (128, 128, 64), (200, 300, 136),
          (512, 4608, 1536), (17, 37, 1024), (300, 1000, 40)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("tile_n", [0, 64, 128, 256])
def test_linear_fused_bias(cuda, M, N, K, tile_n):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(BF)
    b = (torch.randn(N, device=cuda, generator=g) * 0.1).to(BF)
    out = ops.linear(x, w, b, tile_n=tile_n)
    torch.cuda.synchronize()
    ref = ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, _lib.ACT_NONE)
    close(out, ref)
    assert ops.device_error() == 0


@pytest.mark.parametrize("act", [_lib.ACT_RELU, _lib.ACT_SILU, _lib.ACT_SWISH])
@pytest.mark.parametrize("bias_mode", [_lib.BIAS_NONE, _lib.BIAS_FUSED, _lib.BIAS_POST_ROUND])
def test_activation_and_bias_modes(cuda, act, bias_mode):
    g = torch.Generator(device=cuda).manual_seed(act * 10 + bias_mode)
    M, N, K = 48, 320, 256
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.1).to(BF)
    b = (torch.randn(N, device=cuda, generator=g) * 0.5).to(BF)
    out = ops.linear(x, w, b if bias_mode else None, act=act, bias_mode=bias_mode)
    torch.cuda.synchronize()
    close(out, ref_finish(x.float() @ w.float().t(), b, bias_mode, act))


def test_residual_add_in_place(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    M, N, K = 530, 1536, 1536
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.03).to(BF)
    b = (torch.randn(N, device=cuda, generator=g) * 0.1).to(BF)
    res = torch.randn(M, N, device=cuda, generator=g).to(BF)
    expect = r(ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, 0) + res.float())
    ops.linear(x, w, b, add=res, out=res)  # residual updated in place, like the MSAT blocks
    torch.cuda.synchronize()
    close(res, expect)


def test_swiglu_epilogue(cuda):
    """w12 rows interleaved in groups of [32 gate | 32 up]: out = silu(g) * u."""
    g = torch.Generator(device=cuda).manual_seed(5)
    M, D, Hd = 70, 512, 384
    x = torch.randn(M, D, device=cuda, generator=g).to(BF)
    w12 = (torch.randn(2 * Hd, D, device=cuda, generator=g) * 0.05).to(BF)
    b12 = (torch.randn(2 * Hd, device=cuda, generator=g) * 0.1).to(BF)
    idx = torch.cat([torch.cat([torch.arange(gi * 32, gi * 32 + 32), Hd + torch.arange(gi * 32, gi * 32 + 32)])
                     for gi in range(Hd // 32)]).to(cuda)
    out = torch.empty(M, Hd, dtype=BF, device=cuda)
    ops.gemm([ops.gemm_desc(x, w12[idx].contiguous(), out, b12[idx].contiguous(), epilogue=_lib.EPI_SWIGLU)])
    torch.cuda.synchronize()
    y = r(x.float() @ w12.float().t() + b12.float())
    x1, x2 = y.chunk(2, dim=-1)
    close(out, r(r(F.silu(x1)) * x2))


def test_category_weights_and_euler(cuda):
    """Per-batch category slabs (CategorySpecificLinear) + Euler update with row remap."""
    g = torch.Generator(device=cuda).manual_seed(9)
    cats, B, rows, K, N = 5, 3, 18, 1024, 32
    x = torch.randn(B * rows, K, device=cuda, generator=g).to(BF)
    W = (torch.randn(cats, K, N, device=cuda, generator=g) * 0.05).to(BF)  # reference layout
    bb = (torch.randn(cats, N, device=cuda, generator=g) * 0.1).to(BF)
    ids = torch.tensor([4, 0, 2], device=cuda, dtype=torch.int64)
    state = torch.randn(B * 16, N, device=cuda, generator=g).to(BF)
    expect = state.float().clone()
    Wt = W.transpose(1, 2).contiguous()  # [cats, N, K]
    d = ops.gemm_desc(x, Wt, state, bb, bias_mode=_lib.BIAS_POST_ROUND, cat_ids=ids, rows_per_cat=rows,
                      epilogue=_lib.EPI_EULER, rows_in=rows, rows_out=16, row_skip=2, dt=0.25)
    ops.gemm([d])
    torch.cuda.synchronize()
    for bi in range(B):
        c = int(ids[bi])
        v = r(r(x[bi * rows:(bi + 1) * rows].float() @ W[c].float()) + bb[c].float())
        v = v[2:]
        expect[bi * 16:(bi + 1) * 16] = r(expect[bi * 16:(bi + 1) * 16] + r(0.25 * v))
    close(state, expect)


def test_grouped_three_streams(cuda):
    """Three independent problems of very different shape in one launch."""
    g = torch.Generator(device=cuda).manual_seed(11)
    descs, refs, outs, keep = [], [], [], []
    for M in (512, 18, 32):
        x = torch.randn(M, 1536, device=cuda, generator=g).to(BF)
        w = (torch.randn(1536, 1536, device=cuda, generator=g) * 0.03).to(BF)
        b = (torch.randn(1536, device=cuda, generator=g) * 0.1).to(BF)
        o = torch.empty(M, 1536, dtype=BF, device=cuda)
        keep += [x, w, b]  # descriptors hold raw pointers: keep the tensors alive
        descs.append(ops.gemm_desc(x, w, o, b))
        refs.append(ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, 0))
        outs.append(o)
    ops.gemm(descs)
    torch.cuda.synchronize()
    for o, ref in zip(outs, refs):
        close(o, ref)


def test_qkv_epilogue_rmsnorm_rope_layout(cuda):
    """QKV + per-head RMSNorm (weight then cast) + interleaved RoPE, scattered into q/k
    [B, H, L, 64] and v^T [B, H, 64, Lp] at the stream's token offset."""
    g = torch.Generator(device=cuda).manual_seed(13)
    B, H, D, n, L, tok_off = 2, 4, 256, 18, 50, 20
    Lp = 56
    x = torch.randn(B * n, D, device=cuda, generator=g).to(BF)
    w = (torch.randn(3 * H * 64, D, device=cuda, generator=g) * 0.05).to(BF)
    b = (torch.randn(3 * H * 64, device=cuda, generator=g) * 0.1).to(BF)
    qn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    kn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    ang = torch.rand(L, 32, device=cuda, generator=g) * 6.28
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    q = torch.zeros(B, H, L, 64, dtype=BF, device=cuda)
    k = torch.zeros_like(q)
    vt = torch.zeros(B, H, 64, Lp, dtype=BF, device=cuda)
    ops.gemm([ops.qkv_desc(x, w, b, qn, kn, cos, sin, q, k, vt, tok_off=tok_off, rows_per_batch=n)])
    torch.cuda.synchronize()
    y = r(x.float() @ w.float().t() + b.float()).view(B, n, 3, H, 64).permute(2, 0, 3, 1, 4)

    def norm_rope(t, wn):
        tn = r(wn.float() * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)))
        c = cos[tok_off:tok_off + n][None, None]
        s = sin[tok_off:tok_off + n][None, None]
        a, bb = tn[..., 0::2], tn[..., 1::2]
        outr = torch.stack([a * c - bb * s, a * s + bb * c], dim=-1).flatten(-2)
        return r(outr)

    close(q[:, :, tok_off:tok_off + n], norm_rope(y[0], qn))
    close(k[:, :, tok_off:tok_off + n], norm_rope(y[1], kn))
    close(vt[..., tok_off:tok_off + n], y[2].transpose(-1, -2))
    assert q[:, :, :tok_off].abs().sum() == 0 and vt[..., tok_off + n:].abs().sum() == 0


def test_bad_arguments_raise(cuda):
    x = torch.randn(16, 60, device=cuda).to(BF)  # K not a multiple of 8
    w = torch.randn(64, 60, device=cuda).to(BF)
    with pytest.raises(_lib.RldxError):
        ops.linear(x, w)
    with pytest.raises(ValueError):
        ops.linear(x.cpu(), w)


# Arrival counters sit in the first bytes of the workspace (one uint32 per split tile, the
# region rounded up to 256 bytes for up to 1536 units).
COUNTER_BYTES = 6144


def _block_like(cuda, seed, hidden=4096):
    """The four projections of one MSAT block for [VL 512 | SA 18 | P 32] at width 1536."""
    g = torch.Generator(device=cuda).manual_seed(seed)
    keep, cases = [], []
    for M in (512, 18, 32):
        x = torch.randn(M, hidden, device=cuda, generator=g).to(BF)
        w = (torch.randn(1536, hidden, device=cuda, generator=g) * 0.02).to(BF)
        b = (torch.randn(1536, device=cuda, generator=g) * 0.1).to(BF)
        res = torch.randn(M, 1536, device=cuda, generator=g).to(BF)
        keep += [x, w, b, res]
        cases.append((x, w, b, res))
    return keep, cases


@pytest.mark.parametrize("hidden", [3072, 4096])
def test_split_k_workspace_matches_reference_and_is_deterministic(cuda, hidden):
    """Grouped long-K GEMM (w3-like, residual epilogue) through the K-split path: close to the
    fp32 reference, bit-identical across calls, counters back at zero.  (At K = 1536 the planner
    runs these shapes on 64-column tiles without splits: see the next test.)"""
    keep, cases = _block_like(cuda, 21 + hidden, hidden)
    outs = [torch.empty(x.shape[0], 1536, dtype=BF, device=cuda) for x, *_ in cases]
    descs = [ops.gemm_desc(x, w, o, b, add=res) for (x, w, b, res), o in zip(cases, outs)]
    need = ops.gemm_workspace_size(descs)
    assert need > COUNTER_BYTES, "the planner should split K for these shapes"
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    ops.gemm(descs, workspace=ws)
    torch.cuda.synchronize()
    first = [o.clone() for o in outs]
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    ops.gemm(descs, workspace=ws)
    torch.cuda.synchronize()
    for o, f in zip(outs, first):
        assert torch.equal(o, f)
    for (x, w, b, res), o in zip(cases, outs):
        ref = r(ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, 0) + res.float())
        close(o, ref)
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    assert ops.device_error() == 0


def test_narrow_launch_prefers_unsplit_64_column_tiles(cuda):
    """The output-projection shape (K = N = 1536 over [VL 512 | SA 18 | P 32]) has 72 tiles of
    128 columns for 148 SMs: the planner fills the SMs with 64-column tiles instead of K splits
    (measured faster on B200), and the result matches the fp32 reference."""
    keep, cases = _block_like(cuda, 77, 1536)
    outs = [torch.empty(x.shape[0], 1536, dtype=BF, device=cuda) for x, *_ in cases]
    descs = [ops.gemm_desc(x, w, o, b, add=res) for (x, w, b, res), o in zip(cases, outs)]
    plan = ops.gemm_plan(descs)
    if plan["ctas"] >= 144:  # the part has the full SM count the plan is tuned for
        assert plan["tile_n"] == 64 and plan["splits"] == 1, plan
    assert ops.gemm_workspace_size(descs) == 0
    ops.gemm(descs)
    torch.cuda.synchronize()
    for (x, w, b, res), o in zip(cases, outs):
        ref = r(ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, 0) + res.float())
        close(o, ref)
    assert ops.device_error() == 0


def test_split_k_swiglu_and_qkv_epilogues(cuda):
    """The K-split reduction feeds the SwiGLU and QKV epilogues like the unsplit path."""
    g = torch.Generator(device=cuda).manual_seed(31)
    M, K, hid = 18, 1536, 4096
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w12 = (torch.randn(2 * hid, K, device=cuda, generator=g) * 0.03).to(BF)
    b12 = (torch.randn(2 * hid, device=cuda, generator=g) * 0.1).to(BF)
    idx = torch.arange(2 * hid, device=cuda).view(2, hid // 32, 32).permute(1, 0, 2).reshape(-1)
    w12i, b12i = w12[idx].contiguous(), b12[idx].contiguous()
    h_ws = torch.empty(M, hid, dtype=BF, device=cuda)
    h_plain = torch.empty_like(h_ws)
    d_ws = [ops.gemm_desc(x, w12i, h_ws, b12i, epilogue=_lib.EPI_SWIGLU)]
    ws = torch.zeros(max(ops.gemm_workspace_size(d_ws), 16), dtype=torch.uint8, device=cuda)
    ops.gemm(d_ws, workspace=ws)
    ops.gemm([ops.gemm_desc(x, w12i, h_plain, b12i, epilogue=_lib.EPI_SWIGLU)])
    torch.cuda.synchronize()
    y = r(x.float() @ w12.float().t() + b12.float())
    x1, x2 = y.chunk(2, dim=-1)
    close(h_ws, r(r(F.silu(x1)) * x2))
    close(h_ws, h_plain.float())

    H, n, L, tok_off, Lp = 24, 18, 40, 10, 40
    wq = (torch.randn(3 * H * 64, K, device=cuda, generator=g) * 0.03).to(BF)
    bq = (torch.randn(3 * H * 64, device=cuda, generator=g) * 0.1).to(BF)
    qn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    kn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    ang = torch.rand(L, 32, device=cuda, generator=g) * 6.28
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    res = []
    for use_ws in (True, False):
        q = torch.zeros(1, H, L, 64, dtype=BF, device=cuda)
        k = torch.zeros_like(q)
        vt = torch.zeros(1, H, 64, Lp, dtype=BF, device=cuda)
        d = [ops.qkv_desc(x, wq, bq, qn, kn, cos, sin, q, k, vt, tok_off=tok_off, rows_per_batch=n)]
        if use_ws:
            ws = torch.zeros(max(ops.gemm_workspace_size(d), 16), dtype=torch.uint8, device=cuda)
            ops.gemm(d, workspace=ws)
        else:
            ops.gemm(d)
        torch.cuda.synchronize()
        res.append((q, k, vt))
    for a, b in zip(res[0], res[1]):
        close(a, b.float())
    assert ops.device_error() == 0


def test_workspace_too_small_runs_unsplit(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(32, 4096, device=cuda, generator=g).to(BF)
    w = (torch.randn(1536, 4096, device=cuda, generator=g) * 0.02).to(BF)
    out = torch.empty(32, 1536, dtype=BF, device=cuda)
    d = [ops.gemm_desc(x, w, out)]
    ws = torch.zeros(64, dtype=torch.uint8, device=cuda)
    ops.gemm(d, workspace=ws)
    torch.cuda.synchronize()
    close(out, r(x.float() @ w.float().t()))


# ---- CTA pairs (cta_group::2 MMAs over 256-row tiles): large launches plan onto them ----

def _pair_linear(cuda, M, N, K, seed, act=_lib.ACT_NONE, add=False):
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(BF)
    b = (torch.randn(N, device=cuda, generator=g) * 0.1).to(BF)
    res = torch.randn(M, N, device=cuda, generator=g).to(BF) if add else None
    out = torch.empty(M, N, dtype=BF, device=cuda)
    d = ops.gemm_desc(x, w, out, b, act=act, add=res)
    plan = ops.gemm_plan([d])
    ops.gemm([d])
    torch.cuda.synchronize()
    ref = ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, act)
    if add:
        ref = r(ref + res.float())
    return plan, out, ref


@pytest.mark.parametrize("M,N,K", [(4096, 2560, 1024), (4000, 2500, 1000), (2304, 4352, 1536)])
def test_pair_tiles_linear(cuda, M, N, K):
    """Ragged M (not a multiple of 256), N (not a multiple of the pair's half tile) and K (not a
    multiple of 64: two-dimensional tensor maps) on CTA pairs."""
    plan, out, ref = _pair_linear(cuda, M, N, K, seed=M + N + K)
    assert plan["pair"] and plan["ctas"] % 2 == 0, plan
    close(out, ref)
    assert ops.device_error() == 0


def test_pair_tiles_activation_and_residual(cuda):
    plan, out, ref = _pair_linear(cuda, 4096, 3072, 512, seed=77, act=_lib.ACT_SILU, add=True)
    assert plan["pair"], plan
    close(out, ref)


def test_pair_tiles_match_single_cta_tiles(cuda):
    """The same problem on CTA pairs and on single CTAs (a fixed tile width keeps single CTAs)."""
    g = torch.Generator(device=cuda).manual_seed(21)
    M, N, K = 4096, 3072, 768
    x = torch.randn(M, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(BF)
    a, b = torch.empty(M, N, dtype=BF, device=cuda), torch.empty(M, N, dtype=BF, device=cuda)
    da, db = ops.gemm_desc(x, w, a), ops.gemm_desc(x, w, b, tile_n=256)
    assert ops.gemm_plan([da])["pair"] and not ops.gemm_plan([db])["pair"]
    ops.gemm([da])
    ops.gemm([db])
    torch.cuda.synchronize()
    close(a, b.float())
    # both accumulate K in the same chunk order in fp32: the roundings agree almost everywhere
    assert (a != b).float().mean().item() < 0.02


def test_pair_tiles_swiglu_epilogue(cuda):
    g = torch.Generator(device=cuda).manual_seed(23)
    M, D, Hd = 2048, 1024, 4096
    x = torch.randn(M, D, device=cuda, generator=g).to(BF)
    w12 = (torch.randn(2 * Hd, D, device=cuda, generator=g) * 0.05).to(BF)
    b12 = (torch.randn(2 * Hd, device=cuda, generator=g) * 0.1).to(BF)
    idx = torch.cat([torch.cat([torch.arange(gi * 32, gi * 32 + 32), Hd + torch.arange(gi * 32, gi * 32 + 32)])
                     for gi in range(Hd // 32)]).to(cuda)
    out = torch.empty(M, Hd, dtype=BF, device=cuda)
    d = ops.gemm_desc(x, w12[idx].contiguous(), out, b12[idx].contiguous(), epilogue=_lib.EPI_SWIGLU)
    assert ops.gemm_plan([d])["pair"]
    ops.gemm([d])
    torch.cuda.synchronize()
    y = r(x.float() @ w12.float().t() + b12.float())
    x1, x2 = y.chunk(2, dim=-1)
    close(out, r(r(F.silu(x1)) * x2))


def test_pair_tiles_grouped_problems(cuda):
    g = torch.Generator(device=cuda).manual_seed(25)
    descs, refs, outs, keep = [], [], [], []
    for M in (4096, 1024, 2000):
        x = torch.randn(M, 1536, device=cuda, generator=g).to(BF)
        w = (torch.randn(1536, 1536, device=cuda, generator=g) * 0.03).to(BF)
        b = (torch.randn(1536, device=cuda, generator=g) * 0.1).to(BF)
        o = torch.empty(M, 1536, dtype=BF, device=cuda)
        keep += [x, w, b]
        descs.append(ops.gemm_desc(x, w, o, b))
        refs.append(ref_finish(x.float() @ w.float().t(), b, _lib.BIAS_FUSED, 0))
        outs.append(o)
    assert ops.gemm_plan(descs)["pair"]
    ops.gemm(descs)
    torch.cuda.synchronize()
    for o, ref in zip(outs, refs):
        close(o, ref)


def test_pair_tiles_qkv_epilogue(cuda):
    """Per-head RMSNorm + RoPE epilogue on CTA pairs: 256 sequences of 50 tokens, 4 heads."""
    g = torch.Generator(device=cuda).manual_seed(27)
    B, H, D, n, L, tok_off = 256, 4, 256, 50, 56, 3
    Lp = 56
    x = torch.randn(B * n, D, device=cuda, generator=g).to(BF)
    w = (torch.randn(3 * H * 64, D, device=cuda, generator=g) * 0.05).to(BF)
    b = (torch.randn(3 * H * 64, device=cuda, generator=g) * 0.1).to(BF)
    qn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    kn = (1 + 0.1 * torch.randn(64, device=cuda, generator=g)).to(BF)
    ang = torch.rand(L, 32, device=cuda, generator=g) * 6.28
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    q = torch.zeros(B, H, L, 64, dtype=BF, device=cuda)
    k = torch.zeros_like(q)
    vt = torch.zeros(B, H, 64, Lp, dtype=BF, device=cuda)
    d = ops.qkv_desc(x, w, b, qn, kn, cos, sin, q, k, vt, tok_off=tok_off, rows_per_batch=n)
    assert ops.gemm_plan([d])["pair"]
    ops.gemm([d])
    torch.cuda.synchronize()
    y = r(x.float() @ w.float().t() + b.float()).view(B, n, 3, H, 64).permute(2, 0, 3, 1, 4)

    def norm_rope(t, wn):
        tn = r(wn.float() * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)))
        c = cos[tok_off:tok_off + n][None, None]
        s = sin[tok_off:tok_off + n][None, None]
        a, bb = tn[..., 0::2], tn[..., 1::2]
        return r(torch.stack([a * c - bb * s, a * s + bb * c], dim=-1).flatten(-2))

    close(q[:, :, tok_off:tok_off + n], norm_rope(y[0], qn))
    close(k[:, :, tok_off:tok_off + n], norm_rope(y[1], kn))
    close(vt[..., tok_off:tok_off + n], y[2].transpose(-1, -2))
    assert ops.device_error() == 0
