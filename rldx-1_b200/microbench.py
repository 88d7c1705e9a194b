"""Kernel microbenchmarks for BASELINE configs 1, 3 and 4 on one GPU.

    python -m rldx_b200.microbench --suite c1    # one 3-stream MSAT block (config 1 shapes), bf16
    python -m rldx_b200.microbench --suite c3    # memory-bound: Qwen3 QK-RMSNorm+RoPE, SwiGLU
    python -m rldx_b200.microbench --suite gemm  # tensor-bound GEMMs of the batched (config 5) path
    python -m rldx_b200.microbench --suite c4    # joint-attention sweep, head_dim 128
    python -m rldx_b200.microbench --suite vlm   # config-5 VLM-shaped prefill (12 Qwen3 layers)
    python -m rldx_b200.microbench --suite all

Each case prints one JSON line: device time per launch group from CUDA events on the launching
stream (warm-up first, a synchronize on both sides), the algorithmic bytes or FLOPs of the
case, and the achieved rate as a fraction of the measured peak in MEASURED_PEAKS.json (the
fallback figures when that file is absent).  Inputs are seeded ~N(0,1) bf16 tensors created on
the device before timing; every C3 operand is larger than the 126 MB L2, and each C4 iteration
reads tensors that the previous iteration evicted when they exceed L2 (smaller ones are
L2-resident, which the line says).

Config 3 (the Qwen3 backbone path: rldx/model/modules/backbone/modeling_qwen3_vl.py:118-122,
366-371): per-head RMSNorm (cast to bf16, then * weight) + rotate-half RoPE of Q and K
[65536 tokens, 16 heads, 128], positions 0..4095 repeated, theta 1e6; algorithmic bytes = each
tensor read once and written once.  SwiGLU silu(gate) * up on [65536, 8960]: gate and up read
once, the product written once.

VLM prefill (the first part of BASELINE config 5): 12 Qwen3 decoder layers (hidden 2048, GQA
16 / 2 x 128, SwiGLU 11008) over 848 tokens (4 frames x 196 patches + 64 text) per observation,
final RMSNorm, seeded random weights and inputs, 1-D RoPE positions 0..847; one call =
B200LLMChain.forward (the whole stack as one CUDA graph).  FLOPs per call = 2 * tokens *
(projection weights) + 2 * B * heads * T^2 * 128 (causal attention, half of the square).

Config 1 on the GPU: one ExpandedDoubleStreamBlock (cognition 256, action 16, physics 16,
hidden 1024, 16 x 64 heads, SwiGLU 2816, seeded N(0, 0.02) weights, ~N(0,1) streams) through
B200ExpandedDoubleStreamBlock, replayed as one CUDA graph of 11 launches, batch 1 (the latency
case) and larger batches (throughput); FLOPs per block = 2 * 288 * 12.58 M (projections) +
4 * 288^2 * 1024 (attention) = 7.74 GFLOP per batch element.

GEMM suite: the large projections of the batched path on their own (plain bf16 store
epilogue): 8192 x 8192 x 2048, the config-5 VLM w12 at 32 observations (27136 x 22016 x 2048),
the config-2 QKV at 256 observations (131072 x 4608 x 1536); ten launches replayed as one CUDA
graph, FLOPs = 2 M N K; the planner's choice (CTA pairs or single CTAs) is in the line, and
torch.matmul (cuBLAS) on the same operands is timed beside it for context.

Config 4: non-causal joint attention over [cognition | physics | action] segments of lengths
(L-48):32:16, 16 heads x 128, batch 1-64; FLOPs = 4 * B * H * L^2 * 128.  torch's
scaled_dot_product_attention on the same q, k, v (the call the reference makes,
blocks.py:866) is timed beside it for context.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch
import torch.nn.functional as F

from . import ops

ROOT = Path(__file__).resolve().parent.parent
BF = torch.bfloat16


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def time_ms(fn, iters: int, warmup: int) -> float:
    """Average device time of fn() over iters calls (CUDA events on the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(iters):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def suite_c3(iters: int, warmup: int):
    dev = torch.device("cuda", torch.cuda.current_device())
    hbm, _, src = peaks()
    g = torch.Generator(device=dev).manual_seed(3)
    T, H, hd = 65536, 16, 128
    q = torch.randn(T, H, hd, device=dev, generator=g).to(BF)
    k = torch.randn(T, H, hd, device=dev, generator=g).to(BF)
    qw = (1 + 0.1 * torch.randn(hd, device=dev, generator=g)).to(BF)
    kw = (1 + 0.1 * torch.randn(hd, device=dev, generator=g)).to(BF)
    pos = (torch.arange(T, device=dev) % 4096).to(torch.int32)
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=dev).float() / hd))
    emb = torch.outer(torch.arange(4096, device=dev).float(), inv)
    emb = torch.cat([emb, emb], dim=-1)
    cos, sin = emb.cos().to(BF), emb.sin().to(BF)
    qo, ko = torch.empty_like(q), torch.empty_like(k)

    def rope():
        ops.qk_rmsnorm_rope(q, qw, pos, cos, sin, out=qo)
        ops.qk_rmsnorm_rope(k, kw, pos, cos, sin, out=ko)

    ms = time_ms(rope, iters, warmup)
    nbytes = 2 * 2 * q.numel() * 2  # Q and K, each read once and written once
    yield {"suite": "c3", "kernel": "qk_rmsnorm_rope_kernel", "case": "Q and K [65536, 16, 128], pos % 4096, theta 1e6",
           "launches": 2, "ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6, "peak_gbs": hbm,
           "frac": nbytes / ms / 1e6 / hbm, "peak_source": src, "l2": "operands 268 MB each > L2"}
    del q, k, qo, ko

    rows, N = 65536, 8960
    x = torch.randn(rows, 2 * N, device=dev, generator=g).to(BF)
    out = torch.empty(rows, N, dtype=BF, device=dev)
    gate, up = x[:, :N], x[:, N:]
    ms = time_ms(lambda: ops.swiglu(gate, up, out=out), iters, warmup)
    nbytes = 3 * rows * N * 2
    yield {"suite": "c3", "kernel": "swiglu_kernel", "case": "silu(gate) * up, [65536, 8960]", "launches": 1,
           "ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6, "peak_gbs": hbm,
           "frac": nbytes / ms / 1e6 / hbm, "peak_source": src, "l2": "operands 1.17 GB each > L2"}


def suite_c4(iters: int, warmup: int, batches=(1, 4, 16, 64), lengths=(288, 544, 1056, 2080, 4128),
             tiles: int = 0):
    dev = torch.device("cuda", torch.cuda.current_device())
    _, tflops, src = peaks()
    H, hd = 16, 128
    for L in lengths:
        segs = [L - 48, 32, 16]
        Lp = (L + 7) // 8 * 8
        for B in batches:
            g = torch.Generator(device=dev).manual_seed(L * 100 + B)
            q = torch.randn(B, H, L, hd, device=dev, generator=g).to(BF)
            k = torch.randn(B, H, L, hd, device=dev, generator=g).to(BF)
            v = torch.randn(B, H, L, hd, device=dev, generator=g).to(BF)
            vt = torch.zeros(B, H, hd, Lp, dtype=BF, device=dev)
            vt[..., :L] = v.transpose(-1, -2)
            outs = [torch.empty(B * n, H * hd, dtype=BF, device=dev) for n in segs]
            ms = time_ms(lambda: ops.joint_attention(q, k, vt, segs, outs=outs, tiles_per_cta=tiles), iters, warmup)
            ms_sdpa = time_ms(lambda: F.scaled_dot_product_attention(q, k, v), iters, warmup)
            flops = 4.0 * B * H * L * L * hd
            resident = 4 * q.numel() * 2 < 100e6
            yield {"suite": "c4", "kernel": "joint_attention_kernel<128>", "L": L, "B": B, "H": H, "head_dim": hd,
                   "segments": segs, "tiles_per_cta": tiles or "auto", "ms": ms, "flops": flops, "tflops": flops / ms / 1e9,
                   "peak_tflops": tflops, "frac": flops / ms / 1e9 / tflops, "peak_source": src,
                   "torch_sdpa_ms": ms_sdpa, "l2": "q/k/v/out L2-resident" if resident else "q/k/v/out > L2"}
            del q, k, v, vt, outs


def suite_vlm(iters: int, warmup: int, batches=(1, 8, 32), layers: int = 12, T: int = 848):
    from types import SimpleNamespace as NS

    from .llm import B200LLMChain

    dev = torch.device("cuda", torch.cuda.current_device())
    _, tflops, src = peaks()
    D, Hq, Hkv, hd, Fd = 2048, 16, 2, 128, 11008
    g = torch.Generator(device=dev).manual_seed(11)

    def w(*shape, mean=0.0, std=0.02):
        return (torch.randn(*shape, device=dev, generator=g) * std + mean).to(BF)

    def lin(o, i):
        return NS(weight=w(o, i), bias=None)

    stack = []
    for _ in range(layers):
        stack.append(NS(
            input_layernorm=NS(weight=w(D, mean=1.0, std=0.1), variance_epsilon=1e-6),
            post_attention_layernorm=NS(weight=w(D, mean=1.0, std=0.1)),
            self_attn=NS(q_proj=lin(Hq * hd, D), k_proj=lin(Hkv * hd, D), v_proj=lin(Hkv * hd, D),
                         o_proj=lin(D, Hq * hd), q_norm=NS(weight=w(hd, mean=1.0, std=0.1)),
                         k_norm=NS(weight=w(hd, mean=1.0, std=0.1))),
            mlp=NS(gate_proj=lin(Fd, D), up_proj=lin(Fd, D), down_proj=lin(D, Fd))))
    norm = NS(weight=w(D, mean=1.0, std=0.1))
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=dev).float() / hd))
    ang = torch.arange(T, device=dev).float()[:, None] * inv[None, :]
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(BF), emb.sin().to(BF)
    ssin = sin.clone()
    ssin[:, : hd // 2] *= -1
    per_token = 2 * (D * (Hq + 2 * Hkv) * hd + Hq * hd * D + 3 * D * Fd) * layers
    for B in batches:
        chain = B200LLMChain(stack, nn_module(norm), cos, ssin)
        x = torch.randn(B, T, D, device=dev, generator=g).to(BF)
        ms = time_ms(lambda: chain(x), iters, warmup)
        flops = per_token * B * T + 2.0 * B * Hq * T * T * hd * layers
        yield {"suite": "vlm", "what": "12 x Qwen3 decoder layer prefill + final norm (one CUDA graph)",
               "B": B, "tokens": T, "layers": layers, "hidden": D, "heads": f"{Hq}/{Hkv}x{hd}", "ffn": Fd,
               "ms": ms, "ms_per_observation": ms / B, "flops": flops, "tflops": flops / ms / 1e9,
               "peak_tflops": tflops, "frac": flops / ms / 1e9 / tflops, "peak_source": src,
               "launches": chain.launches_per_call}
        del chain, x
        torch.cuda.empty_cache()


def c1_block_module(seed: int = 0):
    """A module with the reference ExpandedDoubleStreamBlock's attribute names and config-1
    shapes, seeded N(0, 0.02) weights and biases (RMSNorm scales 1 + N(0, 0.02))."""
    from torch import nn

    g = torch.Generator().manual_seed(seed)
    dim, heads, hd, hid = 1024, 16, 64, 2816

    def lin(i, o):
        m = nn.Linear(i, o)
        with torch.no_grad():
            m.weight.copy_(torch.randn(o, i, generator=g) * 0.02)
            m.bias.copy_(torch.randn(o, generator=g) * 0.02)
        return m

    blk = nn.Module()
    blk.num_heads = heads
    for s in ("sa", "vl", "p"):
        setattr(blk, f"{s}_qkv", lin(dim, 3 * heads * hd))
        setattr(blk, f"{s}_proj", lin(heads * hd, dim))
        mlp = nn.Module()
        mlp.w12, mlp.w3 = lin(dim, 2 * hid), lin(hid, dim)
        setattr(blk, f"{s}_mlp", mlp)
        for qk in ("q", "k"):
            n = nn.Module()
            n.weight = nn.Parameter(1 + 0.02 * torch.randn(hd, generator=g), requires_grad=False)
            setattr(blk, f"{qk}_norm_{s}", n)
    return blk


def suite_c1(iters: int, warmup: int, batches=(1, 8, 64)):
    from .block import B200ExpandedDoubleStreamBlock

    _, tc_peak, kind = peaks()
    dev = torch.device("cuda", 0)
    blk = c1_block_module(0)
    L, hd = 288, 64
    inv = 1.0 / (1e4 ** (torch.arange(0, hd, 2).float() / hd))
    ang = torch.arange(L).float()[:, None] * inv[None, :]
    pe = torch.polar(torch.ones_like(ang), ang)[None].to(dev)
    flops = 2 * L * (1024 * 3072 + 1024 * 1024 + 1024 * 5632 + 2816 * 1024) + 4.0 * L * L * 1024
    for B in batches:
        g = torch.Generator(device=dev).manual_seed(B)
        cog = torch.randn(B, 256, 1024, device=dev, generator=g).to(BF)
        act = torch.randn(B, 16, 1024, device=dev, generator=g).to(BF)
        phys = torch.randn(B, 16, 1024, device=dev, generator=g).to(BF)
        gpu = B200ExpandedDoubleStreamBlock(blk, dev, use_graph=True)
        gpu(act, cog, phys, pe)
        ms = time_ms(gpu.replay, iters * (10 if B == 1 else 1), warmup)
        tf = flops * B / (ms * 1e-3) / 1e12
        yield {"suite": "c1", "what": "one ExpandedDoubleStreamBlock (config-1 shapes), CUDA graph of "
               f"{gpu.launches} launches", "B": B, "us_per_block": round(ms * 1e3, 2),
               "gflop_per_block": round(flops * B / 1e9, 2), "tflops": round(tf, 1),
               "frac_of_peak": round(tf / tc_peak, 3), "peak": f"{tc_peak} TFLOP/s ({kind})",
               "roofline_us": round(flops * B / (tc_peak * 1e12) * 1e6, 2)}


def graph_time_ms(fn, reps: int = 10, iters: int = 10) -> float:
    """Device time of one fn() call: `reps` calls captured in a CUDA graph, replayed `iters` times."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (iters * reps)


def suite_gemm(shapes=((8192, 8192, 2048), (27136, 22016, 2048), (131072, 4608, 1536))):
    _, tc_peak, kind = peaks()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    for M, N, K in shapes:
        x = torch.randn(M, K, device=dev, generator=g).to(BF)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(BF)
        out = torch.empty(M, N, dtype=BF, device=dev)
        d = [ops.gemm_desc(x, w, out)]
        plan = ops.gemm_plan(d)
        ms = graph_time_ms(lambda: ops.gemm(d))
        ms_ref = graph_time_ms(lambda: torch.matmul(x, w.t(), out=out))
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        yield {"suite": "gemm", "M": M, "N": N, "K": K, "plan": plan, "us": round(ms * 1e3, 1),
               "tflops": round(tf, 1), "frac_of_peak": round(tf / tc_peak, 3),
               "peak": f"{tc_peak} TFLOP/s ({kind}, burst)",
               "cublas_tflops": round(2.0 * M * N * K / (ms_ref * 1e-3) / 1e12, 1)}
        del x, w, out


def nn_module(ns):
    """B200LLMChain stores the final norm as a submodule: wrap the weight holder."""
    m = torch.nn.Module()
    m.weight = torch.nn.Parameter(ns.weight, requires_grad=False)
    return m


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--suite", choices=["c1", "c3", "c4", "vlm", "gemm", "all"], default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batches", type=str, default="1,4,16,64")
    ap.add_argument("--lengths", type=str, default="288,544,1056,2080,4128")
    ap.add_argument("--tiles", type=int, default=0, help="query tiles per attention CTA (0: automatic)")
    ap.add_argument("--gemm-shapes", type=str, default="8192x8192x2048,27136x22016x2048,131072x4608x1536",
                    help="MxNxK list of the gemm suite")
    a = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("microbench needs a CUDA device")
    if a.suite in ("c1", "all"):
        for r in suite_c1(a.iters, a.warmup):
            print(json.dumps(r), flush=True)
    if a.suite in ("c3", "all"):
        for r in suite_c3(a.iters, a.warmup):
            print(json.dumps(r), flush=True)
    if a.suite in ("c4", "all"):
        bs = tuple(int(x) for x in a.batches.split(","))
        ls = tuple(int(x) for x in a.lengths.split(","))
        for r in suite_c4(a.iters, a.warmup, bs, ls, a.tiles):
            print(json.dumps(r), flush=True)
    if a.suite in ("gemm", "all"):
        shapes = tuple(tuple(int(v) for v in t.split("x")) for t in a.gemm_shapes.split(","))
        for r in suite_gemm(shapes):
            print(json.dumps(r), flush=True)
    if a.suite in ("vlm", "all"):
        for r in suite_vlm(a.iters, a.warmup):
            print(json.dumps(r), flush=True)
    assert ops.device_error() == 0, "device error flag set"


if __name__ == "__main__":
    main()
