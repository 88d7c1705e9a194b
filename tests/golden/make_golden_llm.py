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

The video-token-compression fixtures (llm_vtc_*.pt) wrap six such layers in the reference's own
LayerWrapper (rldx/model/modules/backbone/layer_wrapper.py, internal_projection=4 as
modeling_vtc.py:158-164 wires it) and run them through the text model's layer loop
(modeling_qwen3_vl.py:1062-1080: each wrapper returns the layer output and the kwargs it
compressed, which the loop carries to the next layer).  They also record the wrapper's
get_removing_indices on a few marker layouts.

Usage:  python tests/golden/make_golden_llm.py [--deepstack-only | --vtc-only]
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


VTC_LAYERS = 6
VISION_START, VISION_END, IMAGE_PAD = 151652, 151653, 151655


def vtc_ids(frames: int, views: int = 1, patches: int = 16, prefix: int = 4, total: int = T) -> torch.Tensor:
    """Prompt ids: `prefix` text ids, then per frame and view an image-start marker, `patches`
    image ids and an image-end marker, then text up to `total` ids."""
    ids = list(range(1000, 1000 + prefix))
    for _ in range(frames * views):
        ids += [VISION_START] + [IMAGE_PAD] * patches + [VISION_END]
    ids += list(range(2000, 2000 + total - len(ids)))
    return torch.tensor(ids[:total], dtype=torch.long)


def vtc_positions(ids: torch.Tensor, batch: int) -> torch.Tensor:
    """[3, B, T] mRoPE ids for the layout of vtc_ids: text and markers advance all three ids,
    each 4 x 4 image block shares its temporal id and spreads height / width over the grid."""
    pos = torch.zeros(3, ids.numel(), dtype=torch.long)
    p, t = 0, 0
    while t < ids.numel():
        if ids[t] == IMAGE_PAD:
            n = 0
            while t + n < ids.numel() and ids[t + n] == IMAGE_PAD:
                pos[0, t + n] = p
                pos[1, t + n] = p + n // 4
                pos[2, t + n] = p + n % 4
                n += 1
            t += n
            p += 4
        else:
            pos[:, t] = p
            p += 1
            t += 1
    return pos[:, None, :].expand(3, batch, ids.numel()).contiguous()


def fixture_vtc(mod, wrapper_mod, dtype, batch):
    """Six layers wrapped in the reference LayerWrapper (compression before layer 4) over three
    frames of 16 image tokens each: the first two frames (rows [4, 40)) become one mean token."""
    import copy

    global CFG
    saved = CFG
    CFG = copy.replace(saved, layers=VTC_LAYERS) if hasattr(copy, "replace") else oq.Qwen3Config(
        **{**vars(saved), "layers": VTC_LAYERS})
    try:
        stack, rotary = reference_stack(mod)
    finally:
        cfg_vtc, CFG = CFG, saved
    oq.init_weights(stack, seed=2025)
    stack = stack.to(dtype).eval()
    wrapped = [wrapper_mod.LayerWrapper(layer, layer_idx=i, internal_projection=4, img_pattern=[VISION_START],
                                        motion_token=1) for i, layer in enumerate(stack.layers)]
    ids = vtc_ids(frames=3)[None].expand(batch, T).contiguous()
    g = torch.Generator().manual_seed(9)
    h0 = torch.randn(batch, T, cfg_vtc.hidden, generator=g).to(dtype)
    position_ids = vtc_positions(ids[0], batch)
    with torch.no_grad():
        cos, sin = rotary(h0, position_ids)
        kw = {"attention_mask": None, "position_ids": position_ids[0], "past_key_values": None,
              "cache_position": torch.arange(T), "position_embeddings": (cos, sin)}
        hidden = []
        h = h0
        for layer in wrapped:  # the text model's loop, modeling_qwen3_vl.py:1062-1080
            out = layer(h, ids, **kw)
            h = out[0]
            for key in ("attention_mask", "position_ids", "past_key_values", "cache_position",
                        "position_embeddings"):
                if key in out[1]:
                    kw[key] = out[1][key]
            hidden.append(h.clone())
        out = stack.norm(h)
        begin, end = wrapped[4].get_removing_indices(h0, ids)
    return {"config": vars(cfg_vtc), "seed": 2025, "dtype": str(dtype), "batch": batch,
            "inputs": {"hidden": h0, "cos": cos, "sin": sin, "input_ids": ids},
            "compress": (4, int(begin[0, 0]), int(end[0, 0])), "hidden": hidden, "out": out}


def vtc_index_cases(wrapper_mod):
    """The wrapper's (begin, end) on marker layouts: several frames, one frame (begin == end: no
    compression), and image-wise encoding with 2 and 3 views per frame (end = the num_views-th
    last marker)."""
    layer = wrapper_mod.LayerWrapper(nn.Identity(), layer_idx=4, internal_projection=4,
                                     img_pattern=[VISION_START], motion_token=1)
    cases = []
    for frames, views, num_views in ((3, 1, None), (1, 1, None), (4, 1, None), (2, 2, 2), (3, 3, 3), (2, 2, None)):
        ids = vtc_ids(frames, views, patches=6, prefix=3, total=3 + frames * views * 8 + 5)[None]
        b, e = layer.get_removing_indices(torch.zeros(1, ids.shape[1], 1), ids, num_views=
                                          [num_views] if num_views is not None else None)
        cases.append({"input_ids": ids, "num_views": num_views, "begin": int(b[0, 0]), "end": int(e[0, 0])})
    return cases


def main():
    mod = import_reference()
    only_ds = "--deepstack-only" in sys.argv
    only_vtc = "--vtc-only" in sys.argv
    wrapper_mod = importlib.import_module("rldx.model.modules.backbone.layer_wrapper")
    for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        for batch in (1, 2):
            if not only_ds and not only_vtc:
                torch.save(fixture(mod, dtype, batch), HERE / f"llm_b{batch}_{dn}.pt")
            if not only_vtc:
                torch.save(fixture_deepstack(mod, dtype, batch), HERE / f"llm_ds_b{batch}_{dn}.pt")
            fx = fixture_vtc(mod, wrapper_mod, dtype, batch)
            if batch == 1:
                fx["index_cases"] = vtc_index_cases(wrapper_mod)
            torch.save(fx, HERE / f"llm_vtc_b{batch}_{dn}.pt")
    for f in sorted(HERE.glob("llm_*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
