"""Host logic of the VLM prefill chain without a GPU: the static compression rows
(rldx_b200.llm.find_compress_rows / find_compress_info) against the reference LayerWrapper's
get_removing_indices on the layouts recorded in tests/golden/llm_vtc_b1_fp32.pt."""

from pathlib import Path
from types import SimpleNamespace as NS

import pytest
import torch

import rldx_b200  # noqa: F401
from rldx_b200.llm import find_compress_info, find_compress_rows

GOLD = Path(__file__).resolve().parent / "golden"


def test_compress_rows_match_reference_marker_search():
    fx = torch.load(GOLD / "llm_vtc_b1_fp32.pt", weights_only=False)
    for case in fx["index_cases"]:
        assert find_compress_rows(case["input_ids"], num_views=case["num_views"]) == \
            (case["begin"], case["end"]), case


def test_compress_info_from_wrapped_layers():
    """The first wrapper whose layer_idx equals internal_projection compresses; one frame
    (begin == end) gives no compression, as in the reference."""
    fx = torch.load(GOLD / "llm_vtc_b2_fp32.pt", weights_only=False)
    ids = fx["inputs"]["input_ids"]
    layers = [NS(layer=None, layer_idx=i, internal_projection=4, img_pattern=[151652]) for i in range(6)]
    ci = find_compress_info(layers, ids)
    assert ci == {"compress_layer_idx": 4, "static_begin": 4, "static_end": 40, "static_out_len": 65}
    assert find_compress_info(layers, ids, n_cog_tokens=8)["static_out_len"] == 73
    one = next(c for c in torch.load(GOLD / "llm_vtc_b1_fp32.pt", weights_only=False)["index_cases"]
               if c["begin"] == c["end"])
    assert find_compress_info(layers, one["input_ids"]) is None
    assert find_compress_info([NS() for _ in range(6)], ids) is None  # no wrapper: no compression


def test_compress_rows_reject_ragged_batches():
    fx = torch.load(GOLD / "llm_vtc_b1_fp32.pt", weights_only=False)
    a, b = fx["index_cases"][0]["input_ids"], fx["index_cases"][2]["input_ids"]
    n = min(a.shape[1], b.shape[1])
    with pytest.raises(ValueError, match="different rows"):
        find_compress_rows(torch.cat([a[:, :n], b[:, :n]]))
    with pytest.raises(ValueError, match="no image-start marker"):
        find_compress_rows(torch.arange(10)[None])
    with pytest.raises(ValueError, match="fewer than num_views"):
        find_compress_rows(fx["index_cases"][1]["input_ids"], num_views=2)
