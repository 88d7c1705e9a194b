"""Pins the memory-module oracle (oracle/memory_oracle.py) against golden vectors produced by
the reference's own TransformerMemory (tests/golden/make_golden_memory.py): token-causal and
block masks, 96-dim heads, batch 1 and 2, fp32 and bf16."""

from pathlib import Path

import pytest
import torch

from oracle import memory_oracle as mo

GOLD = Path(__file__).resolve().parent / "golden"
NAMES = [f"memory_{m}_b{b}_{dt}.pt" for m in ("causal", "block") for b in (1, 2) for dt in ("fp32", "bf16")]


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_memory(name):
    fx = torch.load(GOLD / name, weights_only=False)
    cfg = mo.MemoryConfig(**fx["config"])
    mem = mo.init_weights(mo.TransformerMemory(cfg), seed=fx["seed"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    mem = mem.to(dtype)
    assert float(sum(p.detach().double().abs().sum() for p in mem.parameters())) == \
        pytest.approx(fx["weight_abs_sum"], rel=1e-9)
    out = mem(fx["inputs"])
    if dtype == torch.bfloat16:
        assert torch.equal(out, fx["out"]), (out.float() - fx["out"].float()).abs().max()
    else:
        torch.testing.assert_close(out, fx["out"], rtol=1e-5, atol=1e-5)
