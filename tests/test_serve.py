"""Serve-level installer (rldx_b200.serve): apply_optimization(policy, "B200") puts the native
action head behind model.get_action, as the reference's _apply_path_cd does for its paths.

CPU: installation, path / RTC-mode checks and the get_action input merge.  GPU: a model whose
backbone hands its features through and whose own get_action is the oracle's eager denoise;
the dispatcher's actions match it with the same noise draws, shape drift falls back to (or
raises instead of) the model's own get_action."""

from types import SimpleNamespace

import pytest
import torch
from torch import nn

import rldx_b200  # noqa: F401
from rldx_b200 import serve
from oracle import msat_oracle as om

BF = torch.bfloat16


class FakeRLDX(nn.Module):
    """RLDX.get_action's structure (rldx/model/core/rldx.py:1117-1155) around an oracle head."""

    def __init__(self, head, rtc_mode="none", rtc_delay=0):
        super().__init__()
        self.action_model = head
        self.use_memory = False
        self.config = SimpleNamespace(rtc_inference_mode=rtc_mode, rtc_inference_delay=rtc_delay)
        self.vanilla_calls = 0

    def backbone(self, bi):
        return {"backbone_features": bi["vl"], "backbone_attention_mask": bi.get("mask")}

    def prepare_input(self, inputs):
        bi = {"vl": inputs["vl"], "mask": inputs.get("mask")}
        ai = {"state": inputs["state"], "embodiment_id": inputs["embodiment_id"]}
        if "physics" in inputs:
            ai["physics"] = inputs["physics"]
        return bi, ai

    def get_action(self, inputs=None, **kwargs):
        from transformers import BatchFeature
        inputs = serve._merge_inputs(inputs, kwargs)
        self.vanilla_calls += 1
        head = self.action_model
        vl = inputs["vl"]
        dev = vl.device
        B = vl.shape[0]
        phys = (None, None)
        if head.use_physics:
            p = head.physics
            fut = torch.randn(B, p.physics_fut_len, p.physics_dim, dtype=BF, device=dev)
            phys = (inputs["physics"][:, :p.physics_hist_len].cpu(), fut.cpu())
        noise = torch.randn(B, head.action_horizon, head.action_dim, dtype=BF, device=dev)
        mask = inputs.get("mask")
        out = om.denoise(head.cpu(), vl.cpu(), inputs["state"].cpu(), inputs["embodiment_id"].cpu(),
                         noise.cpu(), *phys, head.num_inference_timesteps,
                         vl_mask=None if mask is None else mask.cpu())
        return BatchFeature({"action_pred": out.to(dev)})


def _cfg(physics):
    return om.MsatHeadConfig(n_vl=24, n_state=1, horizon=8, physics_hist=4, physics_fut=8, dim=128, heads=2,
                             depth=2, depth_single=0 if physics else 2, use_physics=physics,
                             vl_dim=None if physics else 256, mlp_ratio=3.0, out_dim=64, action_dim=16,
                             state_dim=16, dec_hidden=64, physics_dim=13, num_embodiments=3, num_steps=4,
                             max_seq_len=64, pos_emb_len=32)


def test_apply_optimization_installs_dispatcher():
    model = FakeRLDX(om.ActionHead(_cfg(True)))
    orig = model.get_action
    info = serve.apply_optimization(SimpleNamespace(model=model), "b200")
    assert info["path"] == "B200" and info["bake_prefix_len"] == 0
    assert isinstance(model.get_action, serve.B200Dispatcher)
    assert model.get_action._orig_get_action == orig
    with pytest.raises(ValueError):
        serve.apply_optimization(model, "C")


def test_rtc_modes():
    with pytest.raises(ValueError):
        serve.apply_optimization(FakeRLDX(om.ActionHead(_cfg(False)), rtc_mode="guided"))
    info = serve.apply_optimization(FakeRLDX(om.ActionHead(_cfg(False)), rtc_mode="trained", rtc_delay=3))
    assert info["bake_prefix_len"] == 3


def test_merge_inputs():
    assert serve._merge_inputs({"a": 1}, {"b": 2}) == {"a": 1, "b": 2}
    assert serve._merge_inputs(None, {"inputs": {"a": 1}, "action_prefix": 5}) == {"a": 1, "action_prefix": 5}
    assert serve._merge_inputs(None, {"a": 1}) == {"a": 1}
    with pytest.raises(ValueError):
        serve._merge_inputs({"a": 1}, {"a": 2})


def _request(cfg, cuda, B=1, seed=0):
    inp = om.make_inputs(cfg, batch=B, seed=seed, dtype=BF, emb_ids=[1] * B)
    req = {"vl": inp["vl"].to(cuda), "state": inp["state"].to(cuda), "embodiment_id": inp["embodiment_id"].to(cuda)}
    if cfg.use_physics:
        req["physics"] = torch.cat([inp["physics_hist"], inp["physics_noise"]], 1).to(cuda)
    return req


@pytest.mark.gpu
@pytest.mark.parametrize("physics", [True, False])
def test_dispatcher_matches_model_get_action(cuda, physics):
    cfg = _cfg(physics)
    head = om.init_weights(om.ActionHead(cfg), seed=7).to(BF)
    model = FakeRLDX(head)
    req = _request(cfg, cuda)
    torch.manual_seed(11)
    ref = model.get_action(inputs=dict(req))["action_pred"]
    head.to(cuda)
    serve.apply_optimization(model, "B200")
    torch.manual_seed(11)
    out = model.get_action(inputs=dict(req))["action_pred"]
    torch.cuda.synchronize()
    assert model.get_action.calls == 1
    assert (out.float().cpu() - ref.float().cpu()).abs().max().item() <= 2e-2


@pytest.mark.gpu
def test_dispatcher_shape_drift(cuda):
    cfg = _cfg(False)
    head = om.init_weights(om.ActionHead(cfg), seed=3).to(BF).to(cuda)
    model = FakeRLDX(head)
    serve.apply_optimization(model, "B200")
    model.get_action(inputs=_request(cfg, cuda, B=1))
    n0 = model.vanilla_calls
    out = model.get_action(inputs=_request(cfg, cuda, B=2))  # served by the model's own get_action
    assert out["action_pred"].shape[0] == 2 and model.vanilla_calls == n0 + 1
    model2 = FakeRLDX(head)
    serve.apply_optimization(model2, "B200", on_shape_drift="raise")
    model2.get_action(inputs=_request(cfg, cuda, B=1))
    with pytest.raises(serve.ShapeDrift):
        model2.get_action(inputs=_request(cfg, cuda, B=2))


@pytest.mark.gpu
@pytest.mark.parametrize("physics", [True, False])
def test_dispatcher_serves_masked_backbone_tokens(cuda, physics):
    """A request whose backbone_attention_mask hides some tokens is served natively (the VL key
    mask of every block), matching the model's own masked get_action; an all-ones mask is
    dropped like the reference does."""
    cfg = _cfg(physics)
    head = om.init_weights(om.ActionHead(cfg), seed=7).to(BF)
    model = FakeRLDX(head)
    req = _request(cfg, cuda)
    mask = torch.ones(req["vl"].shape[0], cfg.n_vl, dtype=torch.long, device=cuda)
    mask[:, 5:9] = 0
    req["mask"] = mask
    torch.manual_seed(11)
    ref = model.get_action(inputs=dict(req))["action_pred"]
    head.to(cuda)
    serve.apply_optimization(model, "B200")
    n0 = model.vanilla_calls
    torch.manual_seed(11)
    out = model.get_action(inputs=dict(req))["action_pred"]
    torch.cuda.synchronize()
    assert model.get_action.calls == 1 and model.vanilla_calls == n0  # served natively
    assert (out.float().cpu() - ref.float().cpu()).abs().max().item() <= 2e-2


def test_compile_levels_map_to_paths():
    """The reference server's --compile levels (run_rldx_server.py:117) plus `b200`."""
    from rldx_b200 import server

    assert server.parse_compile_level(None) is None
    assert server.parse_compile_level("none") is None
    assert server.parse_compile_level("submodule") == "B"
    assert server.parse_compile_level("fullgraph") == "D"
    assert server.parse_compile_level("b200") == "B200"
    with pytest.raises(ValueError):
        server.parse_compile_level("max")
    with pytest.raises(ValueError, match="guided"):
        server.validate_compile_level("b200", "guided")
    assert server.validate_compile_level("b200", "trained") == "B200"
    assert server.validate_compile_level("submodule", "guided") == "B"


def test_compile_level_b200_installs_the_dispatcher():
    from rldx_b200 import server

    cfg = _cfg(True)
    model = FakeRLDX(om.init_weights(om.ActionHead(cfg), seed=1))
    policy = SimpleNamespace(model=model)
    info = server.apply_compile_level(policy, "b200")
    assert info["path"] == "B200" and isinstance(model.get_action, serve.B200Dispatcher)
    assert server.apply_compile_level(policy, "none") is None
