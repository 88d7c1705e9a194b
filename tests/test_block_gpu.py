"""BASELINE config 1 on the GPU: one 3-stream ExpandedDoubleStreamBlock (cognition 256, action 16,
physics 16, hidden 1024, 16 x 64 heads, SwiGLU 2816) through B200ExpandedDoubleStreamBlock,
against the oracle block run in bf16 on the CPU (the same roundings) and against the fp32 golden
of the reference block (tests/golden/c1_block_fp32.pt)."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from oracle import msat_oracle as om  # noqa: E402
from rldx_b200 import ops  # noqa: E402
from rldx_b200.block import B200ExpandedDoubleStreamBlock  # noqa: E402

BF = torch.bfloat16
GOLDEN = Path(__file__).resolve().parent / "golden" / "c1_block_fp32.pt"


def cos_sim(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def c1_case(batch=1):
    fx = torch.load(GOLDEN)
    blk = om.init_weights(om.ExpandedDoubleStreamBlock(1024, 16, 64, 2816, 2816), seed=fx["seed_weights"])
    g = torch.Generator().manual_seed(fx["seed_inputs"])
    cog = torch.randn(1, 256, 1024, generator=g)
    act = torch.randn(1, 16, 1024, generator=g)
    phys = torch.randn(1, 16, 1024, generator=g)
    if batch > 1:
        extra = torch.Generator().manual_seed(123)
        cog = torch.cat([cog] + [torch.randn(1, 256, 1024, generator=extra) for _ in range(batch - 1)])
        act = torch.cat([act] + [torch.randn(1, 16, 1024, generator=extra) for _ in range(batch - 1)])
        phys = torch.cat([phys] + [torch.randn(1, 16, 1024, generator=extra) for _ in range(batch - 1)])
    pe = om.RoPEEmbedder1D(64, [64], 1e4, 512)(torch.arange(288).view(1, 288, 1))
    return fx, blk, act, cog, phys, pe


@pytest.mark.parametrize("batch", [1, 3])
def test_c1_block_matches_oracle_bf16(cuda, batch):
    fx, blk, act, cog, phys, pe = c1_case(batch)
    ref_blk = blk.to(BF)
    with torch.no_grad():
        ref = ref_blk(act.to(BF), cog.to(BF), phys.to(BF), pe)
    gpu = B200ExpandedDoubleStreamBlock(ref_blk, cuda)
    out = gpu(act.to(cuda, BF), cog.to(cuda, BF), phys.to(cuda, BF), pe.to(cuda))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for name, o, r in zip(("sa", "vl", "p"), out, ref):
        d = (o.float().cpu() - r.float()).abs().max().item()
        scale = max(1.0, r.float().abs().max().item())
        # fp32 sums in another order leave a bf16 ulp or two: 2e-2 of the output magnitude
        assert d <= 2e-2 * scale, (name, d, scale)
        assert cos_sim(o.cpu(), r) >= 0.9999, name


def test_c1_block_near_fp32_reference_and_graph_replay(cuda):
    fx, blk, act, cog, phys, pe = c1_case(1)
    gpu = B200ExpandedDoubleStreamBlock(blk, cuda, use_graph=True)
    args = (act.to(cuda, BF), cog.to(cuda, BF), phys.to(cuda, BF), pe.to(cuda))
    first = gpu(*args)
    again = gpu(*args)
    eager = B200ExpandedDoubleStreamBlock(blk, cuda)(*args)
    torch.cuda.synchronize()
    for a, b, c in zip(first, again, eager):
        assert torch.equal(a, b)  # graph replay is deterministic
        assert torch.equal(a, c)  # the graph holds exactly the eager launches
    proj = torch.randn(1024, 8, generator=torch.Generator().manual_seed(fx["seed_proj"]))
    for name, o in zip(("sa", "vl", "p"), first):
        # bf16 against the fp32 reference block: signatures agree to bf16 precision
        assert cos_sim(o[0].float().cpu() @ proj, fx["signature"][name]) >= 0.999, name
        assert cos_sim(o[0, 0].float().cpu(), fx["first_rows"][name]) >= 0.999, name


def test_config2_blocks_per_layer_cosine_against_fp32(cuda):
    """The north-star tolerance per layer: four ExpandedDoubleStreamBlocks at config-2 widths
    ([VL 512 | SA 18 | P 32], 1536 wide, 24 x 64 heads, SwiGLU 4096); each layer's bf16 output,
    from the bf16-rounded fp32 input of that layer, has cosine >= 0.9999 against the fp32
    reference block, stream by stream."""
    cfg = om.MsatHeadConfig()
    g = torch.Generator().manual_seed(21)
    sa = torch.randn(1, 18, cfg.dim, generator=g)
    vl = torch.randn(1, 512, cfg.dim, generator=g)
    p = torch.randn(1, 32, cfg.dim, generator=g)
    pe = om.RoPEEmbedder1D(64, [64], 1e4, 1024)(torch.arange(562).view(1, 562, 1))
    for layer in range(4):
        blk = om.init_weights(om.ExpandedDoubleStreamBlock(cfg.dim, cfg.heads, 64, cfg.mlp_hidden,
                                                           cfg.vl_mlp_hidden), seed=100 + layer)
        with torch.no_grad():
            ref = blk(sa, vl, p, pe)
        out = B200ExpandedDoubleStreamBlock(blk, cuda)(sa.to(cuda, BF), vl.to(cuda, BF), p.to(cuda, BF),
                                                        pe.to(cuda))
        torch.cuda.synchronize()
        for name, o, r in zip(("sa", "vl", "p"), out, ref):
            c = cos_sim(o.float().cpu(), r)
            assert c >= 0.9999, (layer, name, c)
        sa, vl, p = ref
    assert ops.device_error() == 0
