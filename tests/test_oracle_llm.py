"""Pins the VLM-prefill oracle (oracle/qwen3_oracle.py) against golden vectors produced by the
reference's own Qwen3-VL text decoder layers (tests/golden/make_golden_llm.py): three layers,
GQA 4 / 2 x 128, FFN 688, mRoPE tables of an image grid + text, batch 1 and 2, fp32 and bf16."""

from pathlib import Path

import pytest
import torch

from oracle import qwen3_oracle as oq

GOLD = Path(__file__).resolve().parent / "golden"
NAMES = [f"llm_b{b}_{dt}.pt" for b in (1, 2) for dt in ("fp32", "bf16")]


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_decoder_stack(name):
    fx = torch.load(GOLD / name, weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    stack = stack.to(dtype)
    assert float(sum(p.detach().double().abs().sum() for p in stack.parameters())) == \
        pytest.approx(fx["weight_abs_sum"], rel=1e-9)
    inp = fx["inputs"]
    out, hidden = stack(inp["hidden"], inp["cos"], inp["sin"], return_hidden=True)
    for got, exp in list(zip(hidden, fx["hidden"])) + [(out, fx["out"])]:
        if dtype == torch.bfloat16:
            assert torch.equal(got, exp), (got.float() - exp.float()).abs().max()
        else:
            torch.testing.assert_close(got, exp, rtol=1e-5, atol=1e-5)


def test_rope_tables_of_text_positions():
    """The 1-D tables the oracle builds for text positions equal the reference's mRoPE tables when
    all three position ids agree (the text part of the golden's position layout)."""
    fx = torch.load(GOLD / "llm_b1_fp32.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    pos = torch.arange(8, 8 + 36)
    cos, sin = oq.rope_tables(cfg, pos)
    torch.testing.assert_close(cos, fx["inputs"]["cos"][0, 64:], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(sin, fx["inputs"]["sin"][0, 64:], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", [f"llm_ds_b{b}_{dt}.pt" for b in (1, 2) for dt in ("fp32", "bf16")])
def test_oracle_deepstack_matches_reference(name):
    """Deepstack visual features after layers 0 and 1 on the 64 image tokens, against the
    reference's own _deepstack_process on its decoder layers."""
    fx = torch.load(GOLD / name, weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(dtype)
    inp = fx["inputs"]
    out, hidden = stack(inp["hidden"], inp["cos"], inp["sin"], return_hidden=True,
                        deepstack=inp["deepstack"], deepstack_rows=inp["deepstack_rows"])
    for got, exp in list(zip(hidden, fx["hidden"])) + [(out, fx["out"])]:
        if dtype == torch.bfloat16:
            assert torch.equal(got, exp), (got.float() - exp.float()).abs().max()
        else:
            torch.testing.assert_close(got, exp, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", [f"llm_vtc_b{b}_{dt}.pt" for b in (1, 2) for dt in ("fp32", "bf16")])
def test_oracle_video_token_compression_matches_reference(name):
    """Six layers with the reference's LayerWrapper (compression before layer 4): the rows of the
    two old frames become one mean token, the RoPE rows follow, layers 4 and 5 run on 65 tokens."""
    fx = torch.load(GOLD / name, weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    dtype = torch.bfloat16 if "bf16" in name else torch.float32
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(dtype)
    inp = fx["inputs"]
    begins, ends = oq.find_compress_rows(inp["input_ids"])
    assert (begins[0], ends[0]) == fx["compress"][1:]
    out, hidden = stack(inp["hidden"], inp["cos"], inp["sin"], return_hidden=True, compress=fx["compress"])
    assert [tuple(h.shape) for h in hidden] == [tuple(h.shape) for h in fx["hidden"]]
    for got, exp in list(zip(hidden, fx["hidden"])) + [(out, fx["out"])]:
        if dtype == torch.bfloat16:
            assert torch.equal(got, exp), (got.float() - exp.float()).abs().max()
        else:
            torch.testing.assert_close(got, exp, rtol=1e-5, atol=1e-5)


def test_compress_rows_match_reference_marker_search():
    """find_compress_rows against the wrapper's get_removing_indices on the recorded layouts
    (several frames, one frame, image-wise encoding with 2 and 3 views)."""
    fx = torch.load(GOLD / "llm_vtc_b1_fp32.pt", weights_only=False)
    for case in fx["index_cases"]:
        b, e = oq.find_compress_rows(case["input_ids"], num_views=case["num_views"])
        assert (b[0], e[0]) == (case["begin"], case["end"]), case
