"""Generates the VLM-prefill golden fixtures (llm_*.pt) from the REFERENCE implementation.

Runs only where the reference checkout is available ($RLDX_REFERENCE, by default a
`reference` directory beside this repository).  It imports the reference's vendored Qwen3-VL text model
(rldx/model/modules/backbone/modeling_qwen3_vl.py: Qwen3VLTextDecoderLayer, Qwen3VLTextRMSNorm,
Qwen3VLTextRotaryEmbedding) under stub parent packages (so rldx/__init__.py's HF processor
imports are skipped; transformers 5 lacks the "default" RoPE init the module looks up, so the
script restores transformers 4's formula for it), builds a small stack with transformers' Qwen3VLTextConfig and the "sdpa"
attention the reference runs with, initialises it with oracle.qwen3_oracle.init_weights (the
oracle has the same parameter names, so the same seed gives the same weights) and records the
per-layer hidden states and the final-norm output.  The RoPE tables come from the reference's
own rotary embedding with 3-D (mRoPE) position ids of an image grid followed by text.

Usage:  python tests/golden/make_golden_llm.py [--deepstack-only]
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

from oracle import qwen3_oracle as oq  # noqa: E402

CFG = oq.Qwen3Config(hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=688, layers=3, rms_eps=1e-6,
                     rope_theta=1e6)
T = 100  # an 8 x 8 image grid (64 tokens) followed by 36 text tokens


def import_reference():
    if not (REF / "rldx").is_dir():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    for name in ["rldx", "rldx.model", "rldx.model.modules", "rldx.model.modules.backbone"]:
        m = types.ModuleType(name)
        m.__path__ = [str(REF / name.replace(".", "/"))]
        sys.modules[name] = m
    mod = importlib.import_module("rldx.model.modules.backbone.modeling_qwen3_vl")
    if "default" not in mod.ROPE_INIT_FUNCTIONS:
        # transformers 5 dropped the "default" entry the reference's rotary embedding looks up
        # (modeling_qwen3_vl.py:306); restore transformers 4's definition:
        # inv_freq = 1 / theta^(2i / head_dim), attention scaling 1.
        def _default_rope(config, device=None, seq_len=None):
            params = getattr(config, "rope_parameters", None) or {}
            base = params.get("rope_theta", getattr(config, "rope_theta", 10000.0))
            dim = config.head_dim
            inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).to(device=device, dtype=torch.float) / dim))
            return inv, 1.0

        mod.ROPE_INIT_FUNCTIONS = {**mod.ROPE_INIT_FUNCTIONS, "default": _default_rope}
    return mod


def mrope_positions(batch: int) -> torch.Tensor:
    """[3, B, T] (t, h, w) ids: the image tokens on an 8 x 8 grid at t = 0, then text with all three
    ids equal, continuing after the grid (the Qwen3-VL layout)."""
    ids = torch.zeros(3, T, dtype=torch.long)
    n_img = 64
    ids[1, :n_img] = torch.arange(n_img) // 8
    ids[2, :n_img] = torch.arange(n_img) % 8
    start = 8
    ids[:, n_img:] = torch.arange(start, start + T - n_img)[None, :]
    return ids[:, None, :].expand(3, batch, T).contiguous()


def reference_stack(mod):
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig

    cfg = Qwen3VLTextConfig(hidden_size=CFG.hidden, num_attention_heads=CFG.q_heads,
                            num_key_value_heads=CFG.kv_heads, head_dim=CFG.head_dim,
                            intermediate_size=CFG.ffn, num_hidden_layers=CFG.layers,
                            rms_norm_eps=CFG.rms_eps, rope_theta=CFG.rope_theta, attention_bias=False,
                            hidden_act="silu", max_position_embeddings=4096)
    cfg._attn_implementation = "sdpa"
    # (in transformers 5 rope_scaling and rope_parameters are one dict: keep the theta in it)
    cfg.rope_scaling = {"rope_type": "default", "mrope_section": [24, 20, 20], "rope_theta": CFG.rope_theta}
    stack = nn.Module()
    stack.layers = nn.ModuleList(mod.Qwen3VLTextDecoderLayer(cfg, i) for i in range(CFG.layers))
    stack.norm = mod.Qwen3VLTextRMSNorm(CFG.hidden, eps=CFG.rms_eps)
    rotary = mod.Qwen3VLTextRotaryEmbedding(cfg)
    return stack, rotary


def fixture(mod, dtype, batch):
    stack, rotary = reference_stack(mod)
    oq.init_weights(stack, seed=2024)
    orc = oq.TextStack(CFG)
    res = orc.load_state_dict(stack.state_dict(), strict=True)
    assert not res.missing_keys and not res.unexpected_keys
    stack = stack.to(dtype).eval()
    g = torch.Generator().manual_seed(7)
    h0 = torch.randn(batch, T, CFG.hidden, generator=g).to(dtype)
    with torch.no_grad():
        cos, sin = rotary(h0, mrope_positions(batch))
        hidden = []
        h = h0
        for layer in stack.layers:
            h = layer(h, position_embeddings=(cos, sin), attention_mask=None)
            hidden.append(h.clone())
        out = stack.norm(h)
    return {"config": vars(CFG), "seed": 2024, "dtype": str(dtype), "batch": batch,
            "weight_abs_sum": float(sum(p.detach().double().abs().sum() for p in stack.parameters())),
            "inputs": {"hidden": h0, "cos": cos, "sin": sin}, "hidden": hidden, "out": out}


def fixture_deepstack(mod, dtype, batch):
    """The same stack with deepstack visual features added after layers 0 and 1 to the 64 image
    tokens of every sequence, through the reference's own Qwen3VLTextModel._deepstack_process
    (modeling_qwen3_vl.py:1086-1113; it reads nothing from the model instance)."""
    stack, rotary = reference_stack(mod)
    oq.init_weights(stack, seed=2024)
    stack = stack.to(dtype).eval()
    g = torch.Generator().manual_seed(8)
    h0 = torch.randn(batch, T, CFG.hidden, generator=g).to(dtype)
    feats = torch.randn(2, 64, CFG.hidden, generator=g).to(dtype)
    mask = torch.zeros(batch, T, dtype=torch.bool)
    mask[:, :64] = True
    with torch.no_grad():
        cos, sin = rotary(h0, mrope_positions(batch))
        hidden = []
        h = h0
        for i, layer in enumerate(stack.layers):
            h = layer(h, position_embeddings=(cos, sin), attention_mask=None)
            if i < feats.shape[0]:
                embeds = feats[i].repeat(batch, 1)  # mask order: sequence by sequence
                h = mod.Qwen3VLTextModel._deepstack_process(None, h, mask, embeds)
            hidden.append(h.clone())
        out = stack.norm(h)
    return {"config": vars(CFG), "seed": 2024, "dtype": str(dtype), "batch": batch,
            "inputs": {"hidden": h0, "cos": cos, "sin": sin, "deepstack": feats,
                       "deepstack_rows": torch.arange(64)},
            "hidden": hidden, "out": out}


def main():
    mod = import_reference()
    only_ds = "--deepstack-only" in sys.argv
    for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        for batch in (1, 2):
            if not only_ds:
                torch.save(fixture(mod, dtype, batch), HERE / f"llm_b{batch}_{dn}.pt")
            torch.save(fixture_deepstack(mod, dtype, batch), HERE / f"llm_ds_b{batch}_{dn}.pt")
    for f in sorted(HERE.glob("llm_*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
