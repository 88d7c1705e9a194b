"""CPU oracle of the memory module (TransformerMemory).

TEST INFRASTRUCTURE ONLY: the checker for the memory variant of rldx_llm_*
(rldx-1_b200/csrc/llm.cu).  Only tests/ and bench.py's CPU baseline may import it.

Restates rldx/model/modules/memory.py step for step, with its module tree and parameter names
so a reference state_dict loads with strict=True:
  RotaryEmbedding          :22-41   fp32 angles, cos / sin cast to the activation dtype
  rotate_half / RoPE       :44-58   q * cos + rotate_half(q) * sin in the activation dtype
  MultiHeadAttention       :61-130  no q / k norm; repeat_interleave for GQA; SDPA with the
                                    additive mask, default scale 1 / sqrt(head_dim)
  SwiGLUMLP                :133-147
  TransformerDecoderLayer  :150-182
  _make_causal_mask        :185-227 finfo.min above the diagonal (or per block)
  TransformerMemory        :230-370 position ids = token // block_attn_size; final RMSNorm
and the shared RMSNorm of rldx/model/modules/norms.py:7-22 (weight times the fp32 normalised
value, then the cast).  Pinned against the reference's own TransformerMemory:
tests/golden/make_golden_memory.py.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class MemoryConfig:
    """TransformerMemory defaults (memory.py:237-251) with BASELINE config 5's memory length:
    8 sets of 256 cognition tokens, hidden 1536 (16 heads of 96), SwiGLU 6144, 2 layers."""

    hidden: int = 1536
    ffn: int = 6144
    layers: int = 2
    heads: int = 16
    kv_heads: int = 16
    rms_eps: float = 1e-5
    block: int = 256        # block_attn_size = tokens per cognition set
    sets: int = 8           # memory_length
    use_causal_attn: bool = True
    rope_base: float = 10000.0

    @property
    def tokens(self) -> int:
        return self.block * self.sets


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (self.weight * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps))).to(x.dtype)


class RotaryEmbedding(nn.Module):
    def __init__(self, dim: int, base: float = 10000.0):
        super().__init__()
        inv = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv, persistent=False)

    def forward(self, x, position_ids):
        inv = self.inv_freq[None, :, None].float().expand(position_ids.shape[0], -1, 1)
        freqs = (inv @ position_ids[:, None, :].float()).transpose(1, 2)
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


def rotate_half(x):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


class MultiHeadAttention(nn.Module):
    def __init__(self, c: MemoryConfig):
        super().__init__()
        self.c = c
        self.head_dim = c.hidden // c.heads
        self.q_proj = nn.Linear(c.hidden, c.heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(c.hidden, c.kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(c.hidden, c.kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(c.heads * self.head_dim, c.hidden, bias=False)
        self.rotary_emb = RotaryEmbedding(self.head_dim, c.rope_base)

    def forward(self, x, mask, position_ids):
        B, T, _ = x.shape
        q = self.q_proj(x).view(B, T, self.c.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.c.kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.c.kv_heads, self.head_dim).transpose(1, 2)
        cos, sin = self.rotary_emb(v, position_ids)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        q, k = q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin
        groups = self.c.heads // self.c.kv_heads
        if groups > 1:
            k, v = k.repeat_interleave(groups, dim=1), v.repeat_interleave(groups, dim=1)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0)
        return self.o_proj(o.transpose(1, 2).reshape(B, T, self.c.hidden))


class SwiGLUMLP(nn.Module):
    def __init__(self, c: MemoryConfig):
        super().__init__()
        self.gate_proj = nn.Linear(c.hidden, c.ffn, bias=False)
        self.up_proj = nn.Linear(c.hidden, c.ffn, bias=False)
        self.down_proj = nn.Linear(c.ffn, c.hidden, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, c: MemoryConfig):
        super().__init__()
        self.self_attn = MultiHeadAttention(c)
        self.mlp = SwiGLUMLP(c)
        self.input_layernorm = RMSNorm(c.hidden, c.rms_eps)
        self.post_attention_layernorm = RMSNorm(c.hidden, c.rms_eps)

    def forward(self, h, mask, position_ids):
        h = h + self.self_attn(self.input_layernorm(h), mask, position_ids)
        return h + self.mlp(self.post_attention_layernorm(h))


def causal_mask(T: int, dtype, block: int = 1, use_causal_attn: bool = True) -> torch.Tensor:
    """_make_causal_mask (memory.py:185-227) for one sequence: [T, T] additive."""
    mask = torch.full((T, T), torch.finfo(dtype).min)
    if use_causal_attn:
        idx = torch.arange(T)
        mask.masked_fill_(idx < (idx + 1).view(T, 1), 0)
    else:
        for i in range(0, T, block):
            mask[i:min(i + block, T), :min(i + block, T)] = 0
    return mask.to(dtype)


class TransformerMemory(nn.Module):
    def __init__(self, c: MemoryConfig):
        super().__init__()
        self.c = c
        self.layers = nn.ModuleList(DecoderLayer(c) for _ in range(c.layers))
        self.norm = RMSNorm(c.hidden, c.rms_eps)

    def position_ids(self, batch: int, T: int) -> torch.Tensor:
        return (torch.arange(T) // self.c.block).unsqueeze(0).expand(batch, -1)

    @torch.no_grad()
    def forward(self, inputs_embeds):
        B, T, _ = inputs_embeds.shape
        pos = self.position_ids(B, T)
        mask = causal_mask(T, inputs_embeds.dtype, self.c.block, self.c.use_causal_attn)[None, None].expand(B, 1, T, T)
        h = inputs_embeds
        for layer in self.layers:
            h = layer(h, mask, pos)
        return self.norm(h)


def init_weights(module: nn.Module, seed: int, std: float = 0.02) -> nn.Module:
    """Seeded random init: linear weights ~ N(0, std), norm weights ~ 1 + N(0, 0.1)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
            if "norm" in name:
                p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(p.dtype))
            else:
                p.copy_((torch.randn(p.shape, generator=g) * std).to(p.dtype))
    return module
