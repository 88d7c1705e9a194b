"""Serve-level installer: the B200 action head behind RLDX.get_action.

Mirrors rldx/inference/serve_optimization.py: `apply_optimization(policy, path)` (:547-601)
installs a dispatcher on `policy.model.get_action` the way `_apply_path_cd` (:519-541) installs
its `_CompiledDispatcher` (:260-516), so PolicyRuntime (rldx/inference/policy_runtime.py:412-435)
keeps calling `model.get_action(**collated)` and gets `BatchFeature({"action_pred": actions})`.

Path "B200": the backbone (and the memory module, when the model has one) runs as the model
defines it; the action head -- state encoder, physics history encoder, num_steps x [action /
physics encoders + MSAT + decoders + Euler] -- runs as one native control step on librldx_b200
(rldx_b200.chain).  The chain is built on the first call from the real shapes (weights copied
into the native arena, one CUDA graph captured); the caller's first call must not run under a
CUDA stream capture.

Error behaviour: like the reference dispatcher, a later call whose input shapes differ from the
bound ones is served by the model's own get_action (on_shape_drift="vanilla", the default) or
raises (on_shape_drift="raise").  Failures of the native library always raise: nothing falls back
silently when librldx_b200.so is missing or a kernel reports an error.  rtc_inference_mode
"guided" is rejected as the reference rejects it for its compiled paths (:568-574); "trained"
bakes the prefix length (config.rtc_inference_delay) into the chain and reads the frozen prefix
from the request's `action_prefix`.
"""

from __future__ import annotations

from typing import Any, Optional

import torch
from torch import nn

from .chain import B200ActionHeadChain, B200ExpandedActionHeadChain


def _find_full_model(policy: Any) -> Any:
    """The RLDX model of an RLDXPolicy, or the model itself (serve_optimization.py:51-53)."""
    return getattr(policy, "model", policy)


def _merge_inputs(inputs: Optional[dict], kwargs: dict) -> dict:
    """RLDX.get_action's merge of the wrapped modality dict and top-level keys
    (rldx/model/core/rldx.py:1117-1146): a collision is an error."""
    if inputs is None:
        inner = kwargs.get("inputs")
        if isinstance(inner, dict):
            extras = {k: v for k, v in kwargs.items() if k != "inputs"}
            inputs, kwargs = inner, extras
        else:
            return dict(kwargs)
    collision = set(inputs).intersection(kwargs)
    if collision:
        raise ValueError("get_action: keys collide between `inputs` dict and top-level kwargs: "
                         f"{sorted(collision)}. Pass each key in exactly one place.")
    return {**inputs, **kwargs}


def _get(container: Any, key: str, default=None):
    if isinstance(container, dict):
        return container.get(key, default)
    if hasattr(container, "get"):
        try:
            return container.get(key, default)
        except TypeError:
            pass
    return getattr(container, key, default)


class ShapeDrift(ValueError):
    """Input shapes differ from the ones the native chain was built for."""


class B200Dispatcher:
    """Callable installed as `full_model.get_action` by apply_optimization(policy, "B200")."""

    def __init__(self, full_model: Any, *, bake_prefix_len: int = 0, on_shape_drift: str = "vanilla",
                 use_graph: bool = True):
        if on_shape_drift not in ("vanilla", "raise"):
            raise ValueError("on_shape_drift must be 'vanilla' or 'raise'")
        self.full_model = full_model
        self.action_model = full_model.action_model
        self._orig_get_action = full_model.get_action
        self.bake_prefix_len = int(bake_prefix_len)
        self.on_shape_drift = on_shape_drift
        self.use_graph = use_graph
        physics = getattr(self.action_model, "physics", None)
        self._has_physics = physics is not None and bool(getattr(self.action_model.model, "use_physics", True)) \
            and hasattr(physics, "physics_cond_encoder")
        self._chain = None
        self.calls = 0

    # ------------------------------------------------------------------------------------------
    def _build(self, device) -> nn.Module:
        cls = B200ExpandedActionHeadChain if self._has_physics else B200ActionHeadChain
        return cls(self.action_model, device, num_inference_timesteps=getattr(
            self.action_model, "num_inference_timesteps", None), use_graph=self.use_graph,
            prefix_len=self.bake_prefix_len)

    def __call__(self, inputs: Optional[dict] = None, **kwargs):
        from transformers import BatchFeature

        fm = self.full_model
        merged = _merge_inputs(inputs, kwargs)
        use_memory = bool(getattr(fm, "use_memory", False))
        reset_memory = merged.pop("reset_memory", None) if use_memory else None
        backbone_inputs, action_inputs = fm.prepare_input(merged)
        with torch.no_grad():
            backbone_outputs = fm.backbone(backbone_inputs)
            if use_memory:
                backbone_outputs = fm._apply_memory_inference(backbone_outputs, reset_memory)
        vl = _get(backbone_outputs, "backbone_features")
        # masked backbone tokens: the VL key mask of every block; an all-ones mask is dropped, as
        # get_action_with_features does (rldx/model/core/rldx.py:619-621)
        mask = _get(backbone_outputs, "backbone_attention_mask")
        if mask is not None and bool(torch.as_tensor(mask).all()):
            mask = None
        state = _get(action_inputs, "state")
        emb = _get(action_inputs, "embodiment_id")
        device, dtype = vl.device, torch.bfloat16
        B = vl.shape[0]
        am = self.action_model
        horizon = int(getattr(am, "action_horizon", None) or am.config.action_horizon)
        action_dim = am.action_decoder.layer2.W.shape[2]

        physics_hist = physics_noise = physics_mask = None
        if self._has_physics:
            ph = _get(action_inputs, "physics")
            if ph is None:
                return self._drift(merged, "the physics head needs action_input.physics")
            hist_len, fut_len = am.physics.physics_hist_len, am.physics.physics_fut_len
            physics_hist = ph[:, :hist_len].to(device=device, dtype=dtype)
            physics_mask = _get(action_inputs, "physics_mask")  # PhysicsHead.prepare_inference's attn_mask
            # drawn first, as PhysicsHead.prepare_inference does (physics_head.py:232-268)
            physics_noise = torch.randn(B, fut_len, am.physics.physics_dim, dtype=dtype, device=device)
        init_noise = torch.randn(B, horizon, action_dim, dtype=dtype, device=device)

        prefix = None
        if self.bake_prefix_len > 0:
            src = merged.get("action_prefix")
            if src is None:
                raise RuntimeError("trained-mode chain requires ``action_prefix`` in the request inputs "
                                   "but none was provided")
            src = torch.as_tensor(src).to(device=device, dtype=dtype)
            if src.shape[1] < self.bake_prefix_len:
                raise RuntimeError(f"action_prefix has {src.shape[1]} timesteps but the chain was baked "
                                   f"for prefix_len={self.bake_prefix_len}")
            prefix = src[:, :self.bake_prefix_len].contiguous()

        if self._chain is None:
            self._chain = self._build(device)
        try:
            if self._has_physics:
                actions = self._chain(vl, state, emb, init_noise, physics_hist=physics_hist,
                                      physics_init_noise=physics_noise, prefix_actions=prefix,
                                      vl_attention_mask=mask,
                                      physics_attention_mask=None if physics_mask is None else physics_mask.view(-1))
            else:
                actions = self._chain(vl, state, emb, init_noise, prefix_actions=prefix, vl_attention_mask=mask)
        except ValueError as e:
            if "differ from the bound shapes" in str(e):
                return self._drift(merged, str(e))
            raise
        self.calls += 1
        return BatchFeature({"action_pred": actions})

    def _drift(self, merged: dict, why: str):
        if self.on_shape_drift == "raise":
            raise ShapeDrift(why)
        return self._orig_get_action(merged)


def apply_optimization(policy: Any, path: str = "B200", compile_mode: Optional[str] = None, *,
                       on_shape_drift: str = "vanilla") -> dict:
    """Install the B200 dispatcher on `policy.model.get_action` (serve_optimization.py:547-601).

    Only path "B200" exists here; the reference's paths A-D stay with the reference.
    compile_mode is accepted for signature compatibility (there is nothing to compile)."""
    del compile_mode
    if str(path).upper() != "B200":
        raise ValueError(f"Unknown optimization path: {path!r} (rldx_b200 provides 'B200')")
    full_model = _find_full_model(policy)
    cfg = getattr(full_model, "config", None)
    rtc_mode = getattr(cfg, "rtc_inference_mode", "none") if cfg is not None else "none"
    if rtc_mode == "guided":
        raise ValueError("path 'B200' cannot serve rtc_inference_mode='guided' (it routes a VJP "
                         "through action_prefix); use 'none' or 'trained'")
    bake = int(getattr(cfg, "rtc_inference_delay", 0) or 0) if rtc_mode == "trained" else 0
    dispatcher = B200Dispatcher(full_model, bake_prefix_len=bake, on_shape_drift=on_shape_drift)
    full_model.get_action = dispatcher
    return {"path": "B200", "installed": "B200Dispatcher", "bake_prefix_len": bake,
            "on_shape_drift": on_shape_drift}
