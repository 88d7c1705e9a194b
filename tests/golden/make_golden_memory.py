"""Generates the memory-module golden fixtures (memory_*.pt) from the REFERENCE implementation.

Runs only where the reference checkout is available ($RLDX_REFERENCE, by default a
`reference` directory beside this repository).  It imports the reference's own TransformerMemory
(rldx/model/modules/memory.py) under stub parent packages, with a `diffusers` stand-in that
only supplies the SinusoidalPositionalEmbedding name the module imports (unused with RoPE) and
a stand-in for rldx.utils.dist.rank_zero_print (a print), initialises it with
oracle.memory_oracle.init_weights (same parameter names, same seed, same weights) and records
the output for a small config (hidden 192 = 2 heads x 96, 2 layers, 3 sets of 32 tokens) in
both mask forms, batch 1 and 2, fp32 and bf16.

Usage:  python tests/golden/make_golden_memory.py
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

from oracle import memory_oracle as mo  # noqa: E402


def import_reference():
    if not (REF / "rldx").is_dir():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    d = types.ModuleType("diffusers")
    d.__path__ = []
    models = types.ModuleType("diffusers.models")
    models.__path__ = []
    emb = types.ModuleType("diffusers.models.embeddings")
    emb.SinusoidalPositionalEmbedding = type("SinusoidalPositionalEmbedding", (nn.Module,), {})
    dist = types.ModuleType("rldx.utils.dist")
    dist.rank_zero_print = print
    sys.modules.update({"diffusers": d, "diffusers.models": models, "diffusers.models.embeddings": emb,
                        "rldx.utils.dist": dist})
    for name in ["rldx", "rldx.model", "rldx.model.modules", "rldx.utils"]:
        m = types.ModuleType(name)
        m.__path__ = [str(REF / name.replace(".", "/"))]
        sys.modules[name] = m
    return importlib.import_module("rldx.model.modules.memory")


CFG = dict(hidden=192, ffn=768, layers=2, heads=2, kv_heads=2, rms_eps=1e-5, block=32, sets=3)


def fixture(mod, dtype, batch, causal):
    cfg = mo.MemoryConfig(**CFG, use_causal_attn=causal)
    ref = mod.TransformerMemory(hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=cfg.layers,
                                num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                                max_position_embeddings=cfg.tokens, rms_norm_eps=cfg.rms_eps,
                                use_causal_attn=causal, use_rope=True, block_attn_size=cfg.block)
    mo.init_weights(ref, seed=99)
    orc = mo.TransformerMemory(cfg)
    res = orc.load_state_dict(ref.state_dict(), strict=True)
    assert not res.missing_keys and not res.unexpected_keys
    ref = ref.to(dtype).eval()
    g = torch.Generator().manual_seed(5)
    x = torch.randn(batch, cfg.tokens, cfg.hidden, generator=g).to(dtype)
    with torch.no_grad():
        out = ref(inputs_embeds=x).last_hidden_state
    return {"config": {**CFG, "use_causal_attn": causal}, "seed": 99, "dtype": str(dtype), "batch": batch,
            "weight_abs_sum": float(sum(p.detach().double().abs().sum() for p in ref.parameters())),
            "inputs": x, "out": out}


def main():
    mod = import_reference()
    for causal, cn in ((True, "causal"), (False, "block")):
        for dtype, dn in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
            for batch in (1, 2):
                torch.save(fixture(mod, dtype, batch, causal), HERE / f"memory_{cn}_b{batch}_{dn}.pt")
    for f in sorted(HERE.glob("memory_*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
