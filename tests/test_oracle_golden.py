"""Pins the CPU oracle against golden vectors produced by the reference implementation itself
(tests/golden/make_golden.py): the reference's GraphSafeActionModel loop (batch 1), its eager
loop around the reference modules (batch 2) and one reference ExpandedDoubleStreamBlock at
BASELINE config 1 shapes.  Three topologies: "small" (physics, double blocks only, config 2's
form), "std" (no physics: DoubleStreamBlocks with a wider VL stream + SingleStreamBlocks, the
production no-add-on form) and "physss" (physics with ExpandedSingleStreamBlocks on top)."""

from pathlib import Path

import pytest
import torch

from oracle import msat_oracle as om

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return torch.load(GOLD / name, weights_only=False)


HEADS = [f"head_{tag}_b{b}_{dt}.pt" for tag in ("small", "std", "physss") for b in (1, 2)
         for dt in ("fp32", "bf16")]


@pytest.mark.parametrize("name", HEADS)
def test_oracle_matches_reference_head(name):
    fx = _load(name)
    cfg = om.MsatHeadConfig(**fx["config"])
    head = om.init_weights(om.ActionHead(cfg), seed=fx["seed"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    if dtype == torch.bfloat16:
        head = head.to(torch.bfloat16)  # also turns the complex RoPE tables into cos-only ones
    wsum = float(sum(p.detach().double().abs().sum() for p in head.parameters()))
    assert wsum == pytest.approx(fx["weight_abs_sum"], rel=1e-9)
    assert (not head.model.rope_embedder.freqs_cis_0.is_complex()) == fx["cos_only_rope"]
    inp = fx["inputs"]
    phys = (inp["physics_hist"], inp["physics_noise"]) if cfg.use_physics else (None, None)
    out = om.denoise(head, inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"],
                     *phys, cfg.num_steps)
    ref = fx["actions"]
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    else:  # same torch CPU kernels in the same order: bit-identical
        assert torch.equal(out, ref), (out.float() - ref.float()).abs().max()


@pytest.mark.parametrize("name", [f"head_{tag}_b2_{dt}.pt" for tag in ("small", "std", "physss")
                                  for dt in ("fp32", "bf16")])
def test_oracle_msat_forward_matches_reference(name):
    fx = _load(name)
    cfg = om.MsatHeadConfig(**fx["config"])
    head = om.init_weights(om.ActionHead(cfg), seed=fx["seed"])
    if "bf16" in name:
        head = head.to(torch.bfloat16)
    inp = fx["inputs"]
    B = inp["vl"].shape[0]
    t0 = torch.zeros(B, dtype=inp["vl"].dtype)
    with torch.no_grad():
        sf = head.state_encoder(inp["state"], inp["embodiment_id"])
        af = head.action_encoder(inp["init_noise"], t0, inp["embodiment_id"]) + \
            head.position_embedding(torch.arange(cfg.horizon)).unsqueeze(0)
        if cfg.use_physics:
            pe = torch.cat([head.physics.physics_cond_encoder(inp["physics_hist"]),
                            head.physics.physics_fut_encoder(inp["physics_noise"], t0)], dim=1)
            out = head.model(torch.cat([sf, af], 1), inp["vl"], t0, pe)
        else:
            out = head.model(torch.cat([sf, af], 1), inp["vl"], t0)
    for k in fx["msat_step0"]:
        if "bf16" in name:
            assert torch.equal(out[k], fx["msat_step0"][k])
        else:
            torch.testing.assert_close(out[k], fx["msat_step0"][k], rtol=1e-5, atol=1e-5)


def test_oracle_c1_block_matches_reference():
    """one 3-stream block, fp32, cog 256 / act 16 / phys 16, hidden 1024."""
    fx = _load("c1_block_fp32.pt")
    blk = om.ExpandedDoubleStreamBlock(1024, 16, 64, 2816, 2816)
    om.init_weights(blk, seed=fx["seed_weights"])
    wsum = float(sum(p.detach().double().abs().sum() for p in blk.parameters()))
    assert wsum == pytest.approx(fx["weight_abs_sum"], rel=1e-9)
    g = torch.Generator().manual_seed(fx["seed_inputs"])
    cog = torch.randn(1, 256, 1024, generator=g)
    act = torch.randn(1, 16, 1024, generator=g)
    phys = torch.randn(1, 16, 1024, generator=g)
    rope = om.RoPEEmbedder1D(64, [64], 1e4, 512)
    pe = rope(torch.arange(288).view(1, 288, 1))
    with torch.no_grad():
        sa, vl, p = blk(act, cog, phys, pe)
    proj = torch.randn(1024, 8, generator=torch.Generator().manual_seed(fx["seed_proj"]))
    for k, v in (("sa", sa), ("vl", vl), ("p", p)):
        torch.testing.assert_close(v[0] @ proj, fx["signature"][k], rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(v[0, 0], fx["first_rows"][k], rtol=1e-5, atol=1e-5)
        assert float(v.double().sum()) == pytest.approx(fx["sums"][k], rel=1e-4, abs=1e-2)


def test_rope_cast_to_bf16_keeps_only_cos():
    """The bf16 cast of a module drops the imaginary part of its RoPE tables (the reference
    quirk the kernels reproduce in cos-only mode)."""
    rope = om.RoPEEmbedder1D(64, [16, 48], 1e4, 32).to(torch.bfloat16)
    assert rope.freqs_cis_1.dtype == torch.bfloat16
    ref = om.precompute_freqs_cis(48, 32, 1e4).real.to(torch.bfloat16)
    assert torch.equal(rope.freqs_cis_1, ref)


@pytest.mark.parametrize("name", [f"rtc_{tag}_b1_{dt}.pt" for tag in ("small", "std")
                                  for dt in ("fp32", "bf16")])
def test_oracle_rtc_prefix_matches_reference(name):
    """RTC trained mode (prefix of 3 frozen actions) against the reference GraphSafeActionModel
    with prefix_len=3, physics and standard topologies."""
    fx = _load(name)
    cfg = om.MsatHeadConfig(**fx["config"])
    head = om.init_weights(om.ActionHead(cfg), seed=fx["seed"])
    if "bf16" in name:
        head = head.to(torch.bfloat16)
    inp = fx["inputs"]
    phys = (inp["physics_hist"], inp["physics_noise"]) if cfg.use_physics else (None, None)
    out = om.denoise(head, inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"],
                     *phys, cfg.num_steps, prefix_actions=fx["prefix_actions"])
    assert torch.equal(out[:, :3], fx["prefix_actions"])
    if "bf16" in name:
        assert torch.equal(out, fx["actions"]), (out.float() - fx["actions"].float()).abs().max()
    else:
        torch.testing.assert_close(out, fx["actions"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", [f"masked_{tag}_b2_{dt}.pt" for tag in ("small", "std", "physss")
                                  for dt in ("fp32", "bf16")])
def test_oracle_masked_keys_match_reference(name):
    """Masked backbone tokens (and a masked physics stream on the physics topologies): the key
    masks of every block kind (double, expanded double, single, expanded single) against the
    reference modules run with encoder_attention_mask / physics_attention_mask."""
    fx = _load(name)
    cfg = om.MsatHeadConfig(**fx["config"])
    head = om.init_weights(om.ActionHead(cfg), seed=fx["seed"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    if dtype == torch.bfloat16:
        head = head.to(torch.bfloat16)
    inp = fx["inputs"]
    phys = (inp["physics_hist"], inp["physics_noise"]) if cfg.use_physics else (None, None)
    out = om.denoise(head, inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"],
                     *phys, cfg.num_steps, vl_mask=fx["vl_mask"], physics_mask=fx["physics_mask"])
    ref = fx["actions"]
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    else:
        assert torch.equal(out, ref), (out.float() - ref.float()).abs().max()
    # the masks matter: the unmasked control step gives other actions
    free = om.denoise(head, inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"],
                      *phys, cfg.num_steps)
    assert not torch.equal(free, out)
