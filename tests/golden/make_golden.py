"""Generates the golden fixtures in this directory from the REFERENCE implementation.

Runs only where the reference checkout is available ($RLDX_REFERENCE, by default a
`reference` directory beside this repository).  It imports the reference's own modules — MSAT / ExpandedDoubleStreamBlock
(rldx/model/modules/action_model/{msat,blocks,ops}.py), the embodiment MLPs, the physics
encoders and rldx/inference/action_model/model/graph_safe_action_model.py:GraphSafeActionModel
(the reference's graph-safe denoise loop) — with three stand-ins that touch no arithmetic of
the path:
  * a `diffusers` stand-in: ModelMixin = nn.Module, register_to_config = identity, and
    Timesteps / TimestepEmbedding taken from oracle/msat_oracle.py (diffusers==0.35.1 is a
    reference dependency that is not vendored; its two classes are restated there);
  * stub parent packages for rldx, rldx.model, rldx.model.modules and rldx.inference.* so their
    heavy __init__ files (HF processors) are not imported;
  * RLDXConfig is not built (it fails on Python 3.12 + transformers 5); modules are built from
    explicit dimensions.

Weights come from oracle.init_weights(seed) applied to the reference modules; the oracle loads
the same state_dict (parameter names are identical), so the fixtures pin the oracle to the
reference on identical weights and inputs.

Usage:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib
import os
import sys
import types
from pathlib import Path

import torch
from torch import nn

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF = Path(os.environ.get("RLDX_REFERENCE", REPO.parent / "reference"))
sys.path.insert(0, str(REPO))

from oracle import msat_oracle as om  # noqa: E402


def import_reference():
    if not (REF / "rldx").is_dir():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    # the inference package imports its siblings as top-level packages; mirror its
    # rldx/inference/_path.py:setup() for a script under rldx/inference/action_model/
    sys.path.insert(0, str(REF / "rldx" / "inference"))
    sys.path.insert(0, str(REF / "rldx" / "inference" / "action_model"))
    d = types.ModuleType("diffusers")
    d.__path__ = []
    d.ModelMixin = nn.Module
    d.ConfigMixin = type("ConfigMixin", (), {})
    cu = types.ModuleType("diffusers.configuration_utils")
    cu.register_to_config = lambda f: f
    models = types.ModuleType("diffusers.models")
    models.__path__ = []
    emb = types.ModuleType("diffusers.models.embeddings")
    emb.Timesteps = lambda num_channels, flip_sin_to_cos, downscale_freq_shift: om.Timesteps(num_channels)
    emb.TimestepEmbedding = lambda in_channels, time_embed_dim: om.TimestepEmbedding(in_channels, time_embed_dim)
    emb.SinusoidalPositionalEmbedding = type("SinusoidalPositionalEmbedding", (), {})
    att = types.ModuleType("diffusers.models.attention")
    att.Attention = type("Attention", (), {})
    att.FeedForward = type("FeedForward", (), {})
    sys.modules.update({"diffusers": d, "diffusers.configuration_utils": cu, "diffusers.models": models,
                        "diffusers.models.embeddings": emb, "diffusers.models.attention": att})
    for name in ["rldx", "rldx.model", "rldx.model.modules", "rldx.inference",
                 "rldx.inference.action_model", "rldx.inference.action_model.model"]:
        m = types.ModuleType(name)
        m.__path__ = [str(REF / name.replace(".", "/"))]
        sys.modules[name] = m
    mods = types.SimpleNamespace()
    mods.msat = importlib.import_module("rldx.model.modules.action_model.msat")
    mods.blocks = importlib.import_module("rldx.model.modules.action_model.blocks")
    mods.ops = importlib.import_module("rldx.model.modules.action_model.ops")
    mods.ecm = importlib.import_module("rldx.model.modules.embodiment_conditioned_mlp")
    mods.physics_head = importlib.import_module("rldx.model.modules.action_model.physics_head")
    mods.gs = importlib.import_module("rldx.inference.action_model.model.graph_safe_action_model")
    return mods


SMALL = om.MsatHeadConfig(n_vl=24, n_state=1, horizon=8, physics_hist=4, physics_fut=8, dim=128,
                          heads=2, head_dim=64, depth=2, mlp_ratio=3.0, out_dim=64, action_dim=16,
                          state_dim=16, dec_hidden=64, physics_dim=13, num_embodiments=3,
                          num_steps=4, max_seq_len=64, pos_emb_len=32)
# standard topology (no physics): DoubleStreamBlocks [VL | SA] with a wider VL stream, then
# SingleStreamBlocks over [VL_proj | time | SA] (the shape of the production no-add-on model)
STD = om.MsatHeadConfig(**{**vars(SMALL), "use_physics": False, "depth_single": 2, "vl_dim": 256})
# physics topology with ExpandedSingleStreamBlocks above the ExpandedDoubleStreamBlocks
PHYS_SS = om.MsatHeadConfig(**{**vars(SMALL), "depth_single": 2, "vl_dim": 256})


def reference_head(R, cfg: om.MsatHeadConfig):
    """Builds the reference action-head modules for `cfg` (rldx/model/core/rldx.py:43-106)."""
    msat = R.msat.MSAT(num_attention_heads=cfg.heads, attention_head_dim=cfg.head_dim,
                       output_dim=cfg.out_dim, depth_multi_stream=cfg.depth,
                       depth_single_stream=cfg.depth_single, dropout=0.0,
                       positional_embeddings=cfg.positional_embeddings,
                       action_model_max_seq_len=cfg.max_seq_len, sa_dim=cfg.dim, vl_dim=cfg.vl_width,
                       qk_norm="rms_norm", use_swiglu=True, mlp_ratio=cfg.mlp_ratio,
                       temb_type="input_token", pre_norm="layer_norm", rope_theta=cfg.rope_theta,
                       use_physics=cfg.use_physics, physics_dim=cfg.physics_dim if cfg.use_physics else 0)
    head = nn.Module()
    head.model = msat
    head.state_encoder = R.ecm.CategorySpecificMLP(cfg.num_embodiments, cfg.state_dim, cfg.dec_hidden, cfg.dim)
    head.action_encoder = R.ecm.MultiEmbodimentActionEncoder(cfg.action_dim, cfg.dim, cfg.num_embodiments)
    head.action_decoder = R.ecm.CategorySpecificMLP(cfg.num_embodiments, cfg.out_dim, cfg.dec_hidden, cfg.action_dim)
    head.position_embedding = nn.Embedding(cfg.pos_emb_len, cfg.dim)
    head.vlln = nn.Identity()
    if cfg.use_physics:
        delta = list(range(-cfg.physics_hist + 1, 1)) + list(range(1, cfg.physics_fut + 1))
        head.physics = R.physics_head.PhysicsHead(physics_dim=cfg.physics_dim, embed_dim=cfg.dim,
                                                  msat_output_dim=cfg.out_dim, physics_delta_indices=delta,
                                                  physics_use_flow_matching=True, physics_loss_weight=1.0,
                                                  action_horizon=cfg.horizon)
    head.use_physics = cfg.use_physics
    return head


def run_reference_loop(R, head, cfg, inp, prefix_actions=None):
    """The reference's GraphSafeActionModel loop; prefix_actions enables its RTC trained mode
    (prefix_len = prefix_actions.shape[1])."""
    d = 0 if prefix_actions is None else prefix_actions.shape[1]
    common = dict(msat=head.model, state_encoder=head.state_encoder, action_encoder=head.action_encoder,
                  action_decoder=head.action_decoder, position_embedding=head.position_embedding,
                  vlln=head.vlln, n_vl=cfg.n_vl, n_sa_pure=cfg.n_state + cfg.horizon,
                  action_horizon=cfg.horizon, action_dim=cfg.action_dim,
                  num_inference_timesteps=cfg.num_steps, device="cpu", dtype=inp["vl"].dtype,
                  prefix_len=d)
    extra = {"prefix_actions": prefix_actions} if d else {}
    if not cfg.use_physics:
        gs = R.gs.GraphSafeActionModel(**common)
        with torch.no_grad():
            return gs(inp["vl"], inp["state"], inp["embodiment_id"], init_noise=inp["init_noise"], **extra)
    gs = R.gs.GraphSafeActionModel(
        **common, physics_cond_encoder=head.physics.physics_cond_encoder,
        physics_fut_encoder=head.physics.physics_fut_encoder, physics_decoder=head.physics.physics_decoder,
        physics_hist_len=cfg.physics_hist, physics_fut_len=cfg.physics_fut, physics_dim=cfg.physics_dim)
    with torch.no_grad():
        return gs(inp["vl"], inp["state"], inp["embodiment_id"], init_noise=inp["init_noise"],
                  physics_hist=inp["physics_hist"], physics_init_noise=inp["physics_noise"], **extra)


def run_vanilla_loop(head, cfg, inp, vl_mask=None, physics_mask=None):
    """vanilla_action_head_forward (benchmark_action_model.py:50-123) around the reference
    modules; unlike GraphSafeActionModel (whose static RoPE table is built for batch 1) it
    accepts any batch.  vl_mask / physics_mask go to MSAT as encoder_attention_mask /
    physics_attention_mask, as get_action_with_features passes them
    (rldx/model/core/rldx.py:619-621, 660-666)."""
    masks = {}
    if vl_mask is not None:
        masks["encoder_attention_mask"] = vl_mask
    with torch.no_grad():
        dt = 1.0 / cfg.num_steps
        vl, B = inp["vl"], inp["vl"].shape[0]
        sf = head.state_encoder(inp["state"], inp["embodiment_id"])
        pos = head.position_embedding(torch.arange(cfg.horizon)).unsqueeze(0)
        cur = inp["init_noise"].clone()
        if not cfg.use_physics:
            for t in range(cfg.num_steps):
                ts = torch.tensor([t / float(cfg.num_steps)], dtype=vl.dtype).expand(B)
                af = head.action_encoder(cur, ts, inp["embodiment_id"]) + pos
                mo = head.model(hidden_states=torch.cat([sf, af], 1), encoder_hidden_states=vl, timestep=ts,
                                **masks)
                cur = cur + dt * head.action_decoder(mo, inp["embodiment_id"])[:, -cfg.horizon:]
            return cur
        phys = head.physics
        hist = phys.physics_cond_encoder(inp["physics_hist"])
        fut = inp["physics_noise"].clone()
        for t in range(cfg.num_steps):
            ts = torch.tensor([t / float(cfg.num_steps)], dtype=vl.dtype).expand(B)
            af = head.action_encoder(cur, ts, inp["embodiment_id"]) + pos
            pe = torch.cat([hist, phys.physics_fut_encoder(fut, ts)], dim=1)
            if physics_mask is not None:
                masks["physics_attention_mask"] = physics_mask
            mo = head.model(hidden_states=torch.cat([sf, af], 1), encoder_hidden_states=vl,
                            timestep=ts, physics_embs=pe, **masks)
            cur = cur + dt * head.action_decoder(mo["action"], inp["embodiment_id"])[:, -cfg.horizon:]
            fut = fut + dt * phys.physics_decoder(mo["physics"][:, -phys.physics_fut_len:])
        return cur


def weight_checksum(module: nn.Module) -> float:
    return float(sum(p.detach().double().abs().sum() for p in module.parameters()))


def head_fixture(R, dtype, batch: int, cfg: om.MsatHeadConfig = SMALL) -> dict:
    """batch 1: the reference GraphSafeActionModel loop; batch > 1: the vanilla eager loop."""
    ref = reference_head(R, cfg)
    om.init_weights(ref, seed=1234)
    orc = om.ActionHead(cfg)
    missing = orc.load_state_dict(ref.state_dict(), strict=True)
    assert not missing.missing_keys and not missing.unexpected_keys
    if dtype == torch.bfloat16:
        ref = ref.to(torch.bfloat16)
    ids = [1] if batch == 1 else [1, 2][:batch]
    inp = om.make_inputs(cfg, batch=batch, seed=42, dtype=dtype, emb_ids=ids)
    if batch == 1:
        actions = run_reference_loop(R, ref, cfg, inp)
    else:
        actions = run_vanilla_loop(ref, cfg, inp)
    # reference-module MSAT call on step-0 inputs, for a per-stream check of the MSAT forward
    with torch.no_grad():
        t0 = torch.zeros(batch, dtype=dtype)
        sf = ref.state_encoder(inp["state"], inp["embodiment_id"])
        af = ref.action_encoder(inp["init_noise"], t0, inp["embodiment_id"]) + \
            ref.position_embedding(torch.arange(cfg.horizon)).unsqueeze(0)
        if cfg.use_physics:
            pe = torch.cat([ref.physics.physics_cond_encoder(inp["physics_hist"]),
                            ref.physics.physics_fut_encoder(inp["physics_noise"], t0)], dim=1)
            msat_out = ref.model(hidden_states=torch.cat([sf, af], 1), encoder_hidden_states=inp["vl"],
                                 timestep=t0, physics_embs=pe)
        else:
            msat_out = {"action": ref.model(hidden_states=torch.cat([sf, af], 1),
                                            encoder_hidden_states=inp["vl"], timestep=t0)}
    return {"config": vars(cfg), "seed": 1234, "weight_abs_sum": weight_checksum(ref),
            "dtype": str(dtype), "batch": batch, "loop": "graph_safe" if batch == 1 else "vanilla",
            "inputs": inp, "actions": actions,
            "msat_step0": {k: v.clone() for k, v in msat_out.items()},
            "cos_only_rope": bool(not ref.model.rope_embedder.freqs_cis_0.is_complex())}


def masked_fixture(R, dtype, cfg: om.MsatHeadConfig) -> dict:
    """Masked backbone tokens (and, on the physics topologies, a masked physics stream) at batch
    2 through the vanilla loop: observation 0 hides VL tokens 3, 7 and 10..13, observation 1 its
    last 6; physics mask [1, 0]."""
    ref = reference_head(R, cfg)
    om.init_weights(ref, seed=1234)
    if dtype == torch.bfloat16:
        ref = ref.to(torch.bfloat16)
    inp = om.make_inputs(cfg, batch=2, seed=42, dtype=dtype, emb_ids=[1, 2])
    vl_mask = torch.ones(2, cfg.n_vl, dtype=torch.long)
    vl_mask[0, [3, 7, 10, 11, 12, 13]] = 0
    vl_mask[1, -6:] = 0
    physics_mask = torch.tensor([1, 0], dtype=torch.long) if cfg.use_physics else None
    actions = run_vanilla_loop(ref, cfg, inp, vl_mask=vl_mask, physics_mask=physics_mask)
    return {"config": vars(cfg), "seed": 1234, "weight_abs_sum": weight_checksum(ref),
            "dtype": str(dtype), "batch": 2, "loop": "vanilla_masked", "inputs": inp,
            "vl_mask": vl_mask, "physics_mask": physics_mask, "actions": actions}


def rtc_fixture(R, dtype, cfg: om.MsatHeadConfig, prefix_len: int = 3) -> dict:
    """RTC trained mode: the reference GraphSafeActionModel(prefix_len=3) loop at batch 1 with a
    seeded frozen prefix (graph_safe_action_model.py:196-300)."""
    ref = reference_head(R, cfg)
    om.init_weights(ref, seed=1234)
    if dtype == torch.bfloat16:
        ref = ref.to(torch.bfloat16)
    inp = om.make_inputs(cfg, batch=1, seed=42, dtype=dtype, emb_ids=[1])
    g = torch.Generator().manual_seed(77)
    prefix = (0.5 * torch.randn(1, prefix_len, cfg.action_dim, generator=g)).to(dtype)
    actions = run_reference_loop(R, ref, cfg, inp, prefix_actions=prefix)
    return {"config": vars(cfg), "seed": 1234, "weight_abs_sum": weight_checksum(ref),
            "dtype": str(dtype), "batch": 1, "loop": "graph_safe_rtc", "inputs": inp,
            "prefix_actions": prefix, "actions": actions}


def c1_block_fixture(R) -> dict:
    """one ExpandedDoubleStreamBlock, fp32, [cog 256 | act 16 | phys 16]."""
    torch.manual_seed(0)
    blk = R.blocks.ExpandedDoubleStreamBlock(
        sa_dim=1024, vl_dim=1024, p_dim=1024, num_attention_heads=16, attention_head_dim=64,
        mlp_ratio=4.125, dropout=0.0, qk_norm="rms_norm", use_swiglu=True,
        positional_embeddings="rope_sa_only", temb_type="input_token", pre_norm="layer_norm")
    om.init_weights(blk, seed=7)
    g = torch.Generator().manual_seed(11)
    cog = torch.randn(1, 256, 1024, generator=g)
    act = torch.randn(1, 16, 1024, generator=g)
    phys = torch.randn(1, 16, 1024, generator=g)
    rope = R.ops.RoPEEmbedder1D(64, [64], 1e4, max_seq_len=512)
    pe = rope(torch.arange(288).view(1, 288, 1))
    with torch.no_grad():
        sa, vl, p = blk(act, cog, None, pe=pe, has_time_token=True, p_tokens=phys)
    proj = torch.randn(1024, 8, generator=torch.Generator().manual_seed(99))
    sig = {k: (v[0] @ proj) for k, v in (("sa", sa), ("vl", vl), ("p", p))}
    return {"seed_weights": 7, "seed_inputs": 11, "seed_proj": 99, "weight_abs_sum": weight_checksum(blk),
            "signature": sig, "first_rows": {"sa": sa[0, 0].clone(), "vl": vl[0, 0].clone(), "p": p[0, 0].clone()},
            "sums": {k: float(v.double().sum()) for k, v in (("sa", sa), ("vl", vl), ("p", p))}}


def main():
    R = import_reference()
    for tag, cfg in (("small", SMALL), ("std", STD), ("physss", PHYS_SS)):
        for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
            torch.save(masked_fixture(R, dtype, cfg), HERE / f"masked_{tag}_b2_{dn}.pt")
    if "--masked-only" in sys.argv:
        return
    for tag, cfg in (("small", SMALL), ("std", STD)):
        for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
            torch.save(rtc_fixture(R, dtype, cfg), HERE / f"rtc_{tag}_b1_{dn}.pt")
    if "--rtc-only" in sys.argv:
        return
    torch.save(head_fixture(R, torch.float32, 1), HERE / "head_small_b1_fp32.pt")
    torch.save(head_fixture(R, torch.bfloat16, 1), HERE / "head_small_b1_bf16.pt")
    torch.save(head_fixture(R, torch.float32, 2), HERE / "head_small_b2_fp32.pt")
    torch.save(head_fixture(R, torch.bfloat16, 2), HERE / "head_small_b2_bf16.pt")
    torch.save(c1_block_fixture(R), HERE / "c1_block_fp32.pt")
    for tag, cfg in (("std", STD), ("physss", PHYS_SS)):
        for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
            for batch in (1, 2):
                torch.save(head_fixture(R, dtype, batch, cfg), HERE / f"head_{tag}_b{batch}_{dn}.pt")
    for f in sorted(HERE.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
