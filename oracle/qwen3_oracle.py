"""CPU oracle of the VLM backbone prefill: a stack of Qwen3 text decoder layers.

TEST INFRASTRUCTURE ONLY: the checker for rldx_llm_* (rldx-1_b200/csrc/llm.cu).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline may import it; the product path never does.

Restates rldx/model/modules/backbone/modeling_qwen3_vl.py (the reference's vendored Qwen3-VL
text model) step for step, with its module tree and parameter names so a reference state_dict
loads with strict=True:
  Qwen3VLTextRMSNorm        :357-374  fp32 variance, cast to the input dtype, then * weight
  rotate_half               :118-122
  apply_rotary_pos_emb      :377-401  q * cos + rotate_half(q) * sin in the input dtype
  Qwen3VLTextAttention      :404-490  per-head q/k RMSNorm before RoPE; sdpa with GQA, causal
  Qwen3VLTextMLP            :493-506  down(silu(gate(x)) * up(x)), no biases
  Qwen3VLTextDecoderLayer   :509-560  pre-norm residual blocks
and the video-token compression of the VTC backbone, rldx/model/modules/backbone/layer_wrapper.py
(LayerWrapper, wrapped around every text layer with internal_projection=4 by modeling_vtc.py:158-164):
  get_removing_indices      :25-51    first / last (or num_views-th last) image-start marker
  forward                   :73-113   before layer `internal_projection`, the rows [begin, end)
                                      become one mean row; RoPE rows follow (:201-240)
The attention call is transformers' sdpa_attention_forward for a causal prefill without a mask:
F.scaled_dot_product_attention(q, k, v, scale=head_dim**-0.5, is_causal=True, enable_gqa=True).
Pinned against golden vectors of the reference's own layers: tests/golden/make_golden_llm.py.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class Qwen3Config:
    """VLM-shaped decoder dims (BASELINE config 5 defaults: hidden 2048, GQA 16 / 2 x 128, FFN 11008)."""

    hidden: int = 2048
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 128
    ffn: int = 11008
    layers: int = 12
    rms_eps: float = 1e-6
    rope_theta: float = 1e6


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps

    def forward(self, x):
        dt = x.dtype
        h = x.to(torch.float32)
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return self.weight * h.to(dt)


def rotate_half(x):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q, k, cos, sin):
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


class Attention(nn.Module):
    def __init__(self, c: Qwen3Config):
        super().__init__()
        self.c = c
        self.head_dim = c.head_dim
        self.scaling = c.head_dim ** -0.5
        self.q_proj = nn.Linear(c.hidden, c.q_heads * c.head_dim, bias=False)
        self.k_proj = nn.Linear(c.hidden, c.kv_heads * c.head_dim, bias=False)
        self.v_proj = nn.Linear(c.hidden, c.kv_heads * c.head_dim, bias=False)
        self.o_proj = nn.Linear(c.q_heads * c.head_dim, c.hidden, bias=False)
        self.q_norm = RMSNorm(c.head_dim, c.rms_eps)
        self.k_norm = RMSNorm(c.head_dim, c.rms_eps)

    def forward(self, x, cos, sin):
        B, T, _ = x.shape
        shape = (B, T, -1, self.head_dim)
        q = self.q_norm(self.q_proj(x).view(shape)).transpose(1, 2)
        k = self.k_norm(self.k_proj(x).view(shape)).transpose(1, 2)
        v = self.v_proj(x).view(shape).transpose(1, 2)
        q, k = apply_rope(q, k, cos, sin)
        o = F.scaled_dot_product_attention(q, k, v, scale=self.scaling, is_causal=T > 1, enable_gqa=True)
        return self.o_proj(o.transpose(1, 2).reshape(B, T, -1))


class MLP(nn.Module):
    def __init__(self, c: Qwen3Config):
        super().__init__()
        self.gate_proj = nn.Linear(c.hidden, c.ffn, bias=False)
        self.up_proj = nn.Linear(c.hidden, c.ffn, bias=False)
        self.down_proj = nn.Linear(c.ffn, c.hidden, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, c: Qwen3Config):
        super().__init__()
        self.self_attn = Attention(c)
        self.mlp = MLP(c)
        self.input_layernorm = RMSNorm(c.hidden, c.rms_eps)
        self.post_attention_layernorm = RMSNorm(c.hidden, c.rms_eps)

    def forward(self, h, cos, sin):
        h = h + self.self_attn(self.input_layernorm(h), cos, sin)
        return h + self.mlp(self.post_attention_layernorm(h))


class TextStack(nn.Module):
    """`layers` decoder layers and the final norm (the text model's `layers` and `norm`)."""

    def __init__(self, c: Qwen3Config):
        super().__init__()
        self.c = c
        self.layers = nn.ModuleList(DecoderLayer(c) for _ in range(c.layers))
        self.norm = RMSNorm(c.hidden, c.rms_eps)

    @torch.no_grad()
    def forward(self, h, cos, sin, final_norm: bool = True, return_hidden: bool = False,
                deepstack=None, deepstack_rows=None, compress=None):
        """deepstack: per-layer visual features [n, D] added, after layer i < len(deepstack), to
        the token rows `deepstack_rows` of every sequence (Qwen3VLTextModel._deepstack_process,
        modeling_qwen3_vl.py:1086-1113: hidden[mask] = hidden[mask] + embeds, one rounding).
        compress: (layer, begin, end) -- video-token compression before that layer (see
        compress_sequence); the returned hidden states are shorter from that layer on."""
        hidden = []
        for i, layer in enumerate(self.layers):
            if compress is not None and i == compress[0] and compress[2] > compress[1]:
                h, cos, sin = compress_sequence(h, cos, sin, compress[1], compress[2])
            h = layer(h, cos, sin)
            if deepstack is not None and i < len(deepstack):
                h = h.clone()
                h[:, deepstack_rows] = h[:, deepstack_rows] + deepstack[i].to(h.dtype)
            hidden.append(h)
        out = self.norm(h) if final_norm else h
        return (out, hidden) if return_hidden else out


def rope_tables(c: Qwen3Config, positions: torch.Tensor, dtype=torch.float32):
    """1-D text RoPE: cos / sin [T, head_dim] of positions (the default rotary embedding with all
    three mRoPE sections on the same position, modeling_qwen3_vl.py:293-354)."""
    inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.int64).float() / c.head_dim))
    freqs = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def init_weights(module: nn.Module, seed: int, std: float = 0.02) -> nn.Module:
    """Seeded random init: linear weights ~ N(0, std), norm weights ~ 1 + N(0, 0.1)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
            if name.endswith("norm.weight") or name.endswith("layernorm.weight") or name == "weight":
                p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(p.dtype))
            else:
                p.copy_((torch.randn(p.shape, generator=g) * std).to(p.dtype))
    return module


def find_compress_rows(input_ids: torch.Tensor, img_pattern=(151652,), num_views=None):
    """(begin, end) token rows of the compressed region of each sequence: begin = the first
    occurrence of `img_pattern` (the image-start marker), end = the last occurrence, or the
    num_views-th last when image-wise encoding keeps the newest frame's views
    (LayerWrapper.get_removing_indices, layer_wrapper.py:25-51).  Returns two lists."""
    n = len(img_pattern)
    pat = torch.tensor(list(img_pattern), dtype=input_ids.dtype)
    begins, ends = [], []
    for row in input_ids:
        hits = [t for t in range(row.numel() - n + 1) if torch.equal(row[t:t + n], pat)]
        if not hits:
            raise ValueError("no image-start marker in the sequence")
        begins.append(hits[0])
        ends.append(hits[-num_views] if num_views is not None else hits[-1])
    return begins, ends


def compress_sequence(h, cos, sin, begin: int, end: int):
    """Video-token compression (LayerWrapper.forward, layer_wrapper.py:73-113, 201-240): the rows
    [begin, end) of every sequence -- the old frames' tokens -- are replaced by one row, their mean,
    placed at `begin`; the rows before and after are kept in order.  The mean is the tensor-dtype
    sum over the sequence axis of the rows weighted 1 (dropped) / 0 (kept), then divided by the
    number of dropped rows, each result rounded to the tensor dtype.  The RoPE rows follow the
    tokens: the mean row takes row `begin`'s cos / sin.  begin, end are shared by the batch (the
    reference inference engine's static indices, graph_safe_qwen3vl_text_model.py:26-59)."""
    T = h.shape[1]
    weight = torch.zeros(T, dtype=h.dtype)
    weight[begin:end] = 1
    total = (h * weight[None, :, None]).sum(dim=1)
    count = torch.full((h.shape[0], 1), end - begin, dtype=torch.int64)
    mean = (total / count).unsqueeze(1)
    h = torch.cat([h[:, :begin], mean, h[:, end:]], dim=1)

    def rows(t):
        return torch.cat([t[:, :begin], t[:, begin:begin + 1], t[:, end:]], dim=1)

    return h, rows(cos), rows(sin)
