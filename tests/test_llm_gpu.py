"""VLM backbone prefill (rldx_llm_*, B200LLMChain) on the GPU against the reference's golden
vectors (tests/golden/llm_*.pt, made by the reference's own Qwen3-VL decoder layers) and against
the pinned oracle at the VLM-shaped dims of BASELINE config 5 (hidden 2048, GQA 16 / 2 x 128,
FFN 11008, 848 tokens)."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200.llm import B200LLMChain  # noqa: E402
from oracle import memory_oracle as om_  # noqa: E402
from oracle import qwen3_oracle as oq  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden"
BF = torch.bfloat16


def signed(sin):
    s = sin.clone()
    s[..., : s.shape[-1] // 2] *= -1
    return s


def cos_sim(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def check_close(out, ref, what):
    """bf16 stack output vs the reference's bf16 eager output: max-abs within 2 % of the output's
    magnitude (2e-2 x max(1, max |ref|)) and cosine >= 0.9999."""
    d = (out.float().cpu() - ref.float().cpu()).abs().max().item()
    scale = max(1.0, ref.float().abs().max().item())
    assert d <= 2e-2 * scale, (what, d, scale)
    assert cos_sim(out.cpu(), ref.cpu()) >= 0.9999, what


@pytest.mark.parametrize("batch", [1, 2])
def test_llm_matches_reference_golden(cuda, batch):
    fx = torch.load(GOLD / f"llm_b{batch}_bf16.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)
    inp = fx["inputs"]
    chain = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda))
    out = chain(inp["hidden"].to(cuda))
    torch.cuda.synchronize()
    check_close(out, fx["out"], "final norm")
    # intermediate: the stack without the final norm equals the last layer's hidden state
    chain2 = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda),
                          apply_final_norm=False)
    h = chain2(inp["hidden"].to(cuda))
    torch.cuda.synchronize()
    check_close(h, fx["hidden"][-1], "last hidden")


@pytest.mark.parametrize("batch", [1, 2])
def test_llm_deepstack_matches_reference_golden(cuda, batch):
    """Deepstack features after layers 0 and 1 on the 64 image tokens (the reference's
    _deepstack_process), passed the way CustomLLMChain takes them: per-layer [n, hidden] features
    and the flat element indices of their rows; repeated calls give the same output."""
    fx = torch.load(GOLD / f"llm_ds_b{batch}_bf16.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)
    inp = fx["inputs"]
    D = cfg.hidden
    rows = inp["deepstack_rows"]
    flat = (rows[:, None] * D + torch.arange(D)[None, :]).reshape(-1).to(cuda)
    feats = [f.to(cuda) for f in inp["deepstack"]]
    chain = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda))
    out = chain(inp["hidden"].to(cuda), deepstack_features=feats, deepstack_flat_indices=flat)
    again = chain(inp["hidden"].to(cuda), deepstack_features=feats, deepstack_flat_indices=flat)
    torch.cuda.synchronize()
    check_close(out, fx["out"], "final norm with deepstack")
    assert torch.equal(out, again)
    plain = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)(inp["hidden"], inp["cos"], inp["sin"])
    assert (out.float().cpu() - plain.float()).abs().max() > 0.1  # the features did change the output
    with pytest.raises(ValueError):
        chain(inp["hidden"].to(cuda))  # bound with deepstack: a call without it is shape drift


def test_llm_config5_shapes_against_oracle(cuda):
    """One layer at the config-5 decoder dims over 848 tokens (784 image + 64 text), batch 2."""
    cfg = oq.Qwen3Config(hidden=2048, q_heads=16, kv_heads=2, head_dim=128, ffn=11008, layers=1)
    stack = oq.init_weights(oq.TextStack(cfg), seed=5).to(BF)
    T = 848
    cos, sin = oq.rope_tables(cfg, torch.arange(T), dtype=BF)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, T, cfg.hidden, generator=g).to(BF)
    ref = stack(x, cos[None], sin[None])
    chain = B200LLMChain(stack.layers, stack.norm, cos.to(cuda), signed(sin).to(cuda))
    out = chain(x.to(cuda))
    torch.cuda.synchronize()
    check_close(out, ref, "config-5 dims")
    # graph replay is deterministic
    out2 = chain(x.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_llm_ffn_not_multiple_of_32(cuda):
    """FFN 688 (not a multiple of 32) is padded with zero rows / columns inside the runtime; the
    golden stack already has it -- here eager launch list == graph."""
    fx = torch.load(GOLD / "llm_b1_bf16.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    assert cfg.ffn % 32 != 0
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)
    inp = fx["inputs"]
    a = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda))
    b = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda),
                     use_graph=False)
    x = inp["hidden"].to(cuda)
    assert torch.equal(a(x), b(x))


@pytest.mark.parametrize("mask", ["causal", "block"])
@pytest.mark.parametrize("batch", [1, 2])
def test_memory_matches_reference_golden(cuda, mask, batch):
    """The memory module (TransformerMemory: 96-dim heads, RoPE without q/k norm, block-wise
    positions, weight-then-cast RMSNorm) against the reference's own module's bf16 output."""
    from oracle import memory_oracle as mo
    from rldx_b200.llm import B200MemoryChain

    fx = torch.load(GOLD / f"memory_{mask}_b{batch}_bf16.pt", weights_only=False)
    cfg = mo.MemoryConfig(**fx["config"])
    mem = mo.init_weights(mo.TransformerMemory(cfg), seed=fx["seed"]).to(BF)
    chain = B200MemoryChain(mem, cuda)
    out = chain(fx["inputs"].to(cuda))
    torch.cuda.synchronize()
    check_close(out, fx["out"], f"memory {mask}")


def test_memory_config5_shapes_against_oracle(cuda):
    """Config-5 memory: 8 sets x 256 tokens, hidden 1536 (16 heads of 96), SwiGLU 6144, 2 layers."""
    from oracle import memory_oracle as mo
    from rldx_b200.llm import B200MemoryChain

    cfg = mo.MemoryConfig()
    mem = mo.init_weights(mo.TransformerMemory(cfg), seed=4).to(BF)
    x = torch.randn(1, cfg.tokens, cfg.hidden, generator=torch.Generator().manual_seed(1)).to(BF)
    ref = mem(x)
    out = B200MemoryChain(mem, cuda)(x.to(cuda))
    torch.cuda.synchronize()
    check_close(out, ref, "config-5 memory")


@pytest.mark.parametrize("concat", [True, False])
def test_memory_cache_over_consecutive_calls(cuda, concat):
    """B200MemoryCache against GraphSafeVLA's sliding-window memory (graph_safe_vla.py:106-140)
    restated on the pinned oracle: three calls in a row (the cache fills set by set), two
    sequences, 40 cognition tokens of which the last 32 enter a 3-set memory."""
    from rldx_b200.llm import B200MemoryCache

    cfg = om_.MemoryConfig(hidden=192, ffn=768, layers=2, heads=2, kv_heads=2, rms_eps=1e-5, block=32, sets=3)
    mem = om_.init_weights(om_.TransformerMemory(cfg), seed=4).to(BF)
    mcfg = {"n_cog_tokens": 40, "memory_n_cog_tokens": 32, "memory_length": 3, "concat_memory": concat,
            "hidden_size": 192}
    dev_cache = B200MemoryCache(mem, mcfg, batch=2, device=cuda)
    cached = torch.zeros(2, 96, 192, dtype=BF)
    g = torch.Generator().manual_seed(12)
    for step in range(3):
        vl = torch.randn(2, 50, 192, generator=g).to(BF)
        cog_all = vl[:, -40:]
        cached = torch.cat([cached[:, 32:], cog_all[:, 8:]], dim=1)
        aug = mem(cached)[:, -32:]
        ref = torch.cat([cog_all, aug], 1) if concat else torch.cat([cog_all[:, :8], aug], 1)
        out = dev_cache(vl.to(cuda))
        torch.cuda.synchronize()
        assert out.shape == ref.shape
        check_close(out, ref, f"step {step}")
    dev_cache.reset_memory()
    assert int(dev_cache._cached_cog.abs().sum().item()) == 0


@pytest.mark.parametrize("batch", [1, 2])
def test_llm_video_token_compression_matches_reference_golden(cuda, batch):
    """Six layers wrapped in the reference's LayerWrapper (compression before layer 4 of the rows
    of the two old frames, tests/golden/make_golden_llm.py): one chain, one graph, 100 tokens in,
    65 out; the compression info comes from the prompt's input_ids as the reference engine
    derives it.  Eager launch list == graph."""
    from rldx_b200.llm import find_compress_info

    fx = torch.load(GOLD / f"llm_vtc_b{batch}_bf16.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)
    inp = fx["inputs"]
    wrapped = [torch.nn.Module() for _ in stack.layers]
    for i, (w, layer) in enumerate(zip(wrapped, stack.layers)):
        w.layer, w.layer_idx, w.internal_projection, w.img_pattern = layer, i, 4, [151652]
    ci = find_compress_info(wrapped, inp["input_ids"])
    assert (ci["compress_layer_idx"], ci["static_begin"], ci["static_end"]) == fx["compress"]
    cos, ssin = inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda)
    chain = B200LLMChain(wrapped, stack.norm, cos, ssin, compress_info=ci)
    out = chain(inp["hidden"].to(cuda))
    torch.cuda.synchronize()
    assert out.shape == fx["out"].shape and chain.out_tokens == 65
    check_close(out, fx["out"], "final norm after compression")
    eager = B200LLMChain(wrapped, stack.norm, cos, ssin, compress_info=ci, use_graph=False)
    assert torch.equal(eager(inp["hidden"].to(cuda)), out)
    last = B200LLMChain(wrapped, stack.norm, cos, ssin, compress_info=ci, apply_final_norm=False)
    h = last(inp["hidden"].to(cuda))
    torch.cuda.synchronize()
    check_close(h, fx["hidden"][-1], "last hidden after compression")
    assert chain.device_status() == 0


@pytest.mark.parametrize("layer,begin,end", [(0, 3, 40), (1, 0, 100), (1, 10, 100), (2, 50, 51)])
def test_llm_compression_edges_against_oracle(cuda, layer, begin, end):
    """Compression before the first layer, of the whole sequence, up to the last row, and of a
    single row (the mean of one row is the row), against the pinned oracle."""
    fx = torch.load(GOLD / "llm_b2_bf16.pt", weights_only=False)
    cfg = oq.Qwen3Config(**fx["config"])
    stack = oq.init_weights(oq.TextStack(cfg), seed=fx["seed"]).to(BF)
    inp = fx["inputs"]
    ref = stack(inp["hidden"], inp["cos"], inp["sin"], compress=(layer, begin, end))
    chain = B200LLMChain(stack.layers, stack.norm, inp["cos"][0].to(cuda), signed(inp["sin"][0]).to(cuda),
                         compress_info={"compress_layer_idx": layer, "static_begin": begin, "static_end": end})
    out = chain(inp["hidden"].to(cuda))
    torch.cuda.synchronize()
    assert out.shape == ref.shape
    check_close(out, ref, f"compress {layer} [{begin}, {end})")


def test_llm_config5_compression_against_oracle(cuda):
    """Config-5 decoder dims with the VTC layout of the bench: 4 frames x (marker + 196 patches +
    marker) after 8 text ids, 48 text ids and 256 cognition tokens (1104 tokens); the first three
    frames are compressed before layer 1 of 2 (511 tokens after)."""
    from rldx_b200.llm import find_compress_rows

    cfg = oq.Qwen3Config(hidden=2048, q_heads=16, kv_heads=2, head_dim=128, ffn=11008, layers=2)
    stack = oq.init_weights(oq.TextStack(cfg), seed=6).to(BF)
    ids = torch.tensor(list(range(8)) + ([151652] + [151655] * 196 + [151653]) * 4 + list(range(48)))
    begin, end = find_compress_rows(ids)
    assert (begin, end) == (8, 8 + 3 * 198)
    T = ids.numel() + 256
    cos, sin = oq.rope_tables(cfg, torch.arange(T), dtype=BF)
    x = torch.randn(1, T, cfg.hidden, generator=torch.Generator().manual_seed(4)).to(BF)
    ref = stack(x, cos[None], sin[None], compress=(1, begin, end))
    chain = B200LLMChain(stack.layers, stack.norm, cos.to(cuda), signed(sin).to(cuda),
                         compress_info={"compress_layer_idx": 1, "static_begin": begin, "static_end": end})
    out = chain(x.to(cuda))
    torch.cuda.synchronize()
    assert out.shape == (1, 511, cfg.hidden)
    check_close(out, ref, "config-5 compression")
