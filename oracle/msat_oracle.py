"""CPU restatement of RLDX-1's all-modality MSAT action head — TEST INFRASTRUCTURE ONLY.

This module is the parity oracle for librldx_b200: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it.  It never runs on the product path.

It restates, in plain torch on the CPU, the reference modules and the denoise loop with the
same module tree and parameter names, so a reference state_dict loads into it unchanged
(tests/golden/make_golden.py pins it against the reference modules that way):

  RMSNorm                      rldx/model/modules/norms.py:7-22
  LayerNorm (no affine)        rldx/model/modules/norms.py:25-40
  precompute_freqs_cis         rldx/model/modules/action_model/ops.py:11-25
  apply_rotary_emb             rldx/model/modules/action_model/ops.py:48-67
  RoPEEmbedder1D               rldx/model/modules/action_model/ops.py:70-119
  TimestepEncoder              rldx/model/modules/action_model/ops.py:123-133
  Timesteps / TimestepEmbedding  diffusers==0.35.1 (not vendored in the reference; restated
                               from its published definition: get_timestep_embedding with
                               flip_sin_to_cos=True, downscale_freq_shift=1; Linear-SiLU-Linear)
  SwiGLUFFN                    rldx/model/modules/action_model/ops.py:137-161
  DoubleStreamBlock            rldx/model/modules/action_model/blocks.py:257-609
  ExpandedDoubleStreamBlock    rldx/model/modules/action_model/blocks.py:612-891 (input_token
                               temb => identity modulation, blocks.py:737-760)
  SingleStreamBlock            rldx/model/modules/action_model/blocks.py:42-254
  ExpandedSingleStreamBlock    rldx/model/modules/action_model/blocks.py:894-1089
  MSAT._forward_inner          rldx/model/modules/action_model/msat.py:291-556 (standard path:
                               DoubleStreamBlocks [VL | SA] -> SingleStreamBlocks [VL_proj | SA])
  MSAT._forward_physics        rldx/model/modules/action_model/msat.py:558-781 (ExpandedDouble
                               [VL | SA | P] -> ExpandedSingle [VL_proj + SA | P])
  CategorySpecificLinear/MLP   rldx/model/modules/embodiment_conditioned_mlp.py:62-164
  MultiEmbodimentActionEncoder rldx/model/modules/embodiment_conditioned_mlp.py:180-227
  SinusoidalPositionalEncoding rldx/model/modules/embodiment_conditioned_mlp.py:29-59
  Physics encoders / decoder   rldx/model/modules/action_model/physics.py:9-70
  denoise loop                 rldx/inference/action_model/benchmark_action_model.py:50-123
                               (vanilla_action_head_forward; same as rldx/model/core/rldx.py:490-735
                               without RTC)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn


# ----------------------------------------------------------------------------------------------
# configuration
# ----------------------------------------------------------------------------------------------
@dataclass
class MsatHeadConfig:
    """Dimensions of the all-modality action head (BASELINE config 2 by default)."""

    n_vl: int = 512
    n_state: int = 1
    horizon: int = 16
    physics_hist: int = 16
    physics_fut: int = 16
    dim: int = 1536  # sa_dim == p_dim == heads * head_dim
    heads: int = 24
    head_dim: int = 64
    depth: int = 16  # double-stream blocks
    depth_single: int = 0  # single-stream blocks after them
    use_physics: bool = True
    vl_dim: Optional[int] = None  # width of the VL stream in the double blocks (None: dim)
    mlp_ratio: float = 4.0
    vl_mlp_ratio: Optional[float] = None
    out_dim: int = 1024  # MSAT output_dim == hidden_size
    action_dim: int = 32
    state_dim: int = 64
    dec_hidden: int = 1024
    physics_dim: int = 37
    num_embodiments: int = 36
    num_steps: int = 4
    positional_embeddings: str = "rope_sa_only"
    rope_theta: float = 10000.0
    max_seq_len: int = 1024  # action_model_max_seq_len (RoPE table length)
    pos_emb_len: int = 1024  # config.max_seq_len (position_embedding rows)

    @property
    def mlp_hidden(self) -> int:
        return int(2 / 3 * int(self.dim * self.mlp_ratio))

    @property
    def vl_width(self) -> int:
        return self.vl_dim if self.vl_dim is not None else self.dim

    @property
    def vl_mlp_hidden(self) -> int:
        r = self.vl_mlp_ratio if self.vl_mlp_ratio is not None else self.mlp_ratio
        return int(2 / 3 * int(self.vl_width * r))

    @property
    def single_expanded(self) -> int:  # SwiGLU width of a single-stream block (w12 out / 2)
        return int(self.dim * self.mlp_ratio)

    @property
    def single_mlp_hidden(self) -> int:  # mlp_proj output width of a single-stream block
        return int(2 / 3 * self.single_expanded)


# ----------------------------------------------------------------------------------------------
# primitives
# ----------------------------------------------------------------------------------------------
class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (self.weight * xn).to(x.dtype)


def _ln(dim: int) -> nn.LayerNorm:
    return nn.LayerNorm(dim, elementwise_affine=False, eps=1e-6)


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0) -> torch.Tensor:
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: (dim // 2)].float() / dim))
    t = torch.arange(end, device=freqs.device)
    freqs = torch.outer(t, freqs).float()
    return torch.polar(torch.ones_like(freqs), freqs)


def apply_rotary_emb(xq, xk, freqs_cis):
    """Interleaved-pair complex rotation; a real (cast) table multiplies both halves by cos."""
    xq_ = torch.view_as_complex(xq.float().reshape(*xq.shape[:-1], -1, 2))
    xk_ = torch.view_as_complex(xk.float().reshape(*xk.shape[:-1], -1, 2))
    fc = freqs_cis.unsqueeze(1)
    xq_out = torch.view_as_real(xq_ * fc).flatten(3)
    xk_out = torch.view_as_real(xk_ * fc).flatten(3)
    return xq_out.type_as(xq), xk_out.type_as(xk)


class RoPEEmbedder1D(nn.Module):
    def __init__(self, head_dim: int, axes_dim: list, theta: float, max_seq_len: int):
        super().__init__()
        assert sum(axes_dim) == head_dim
        self.head_dim = head_dim
        self.theta = theta
        self.max_seq_len = max_seq_len
        self.axes_dim = axes_dim
        self.n_axes = len(axes_dim)
        for i, d in enumerate(axes_dim):
            self.register_buffer(f"freqs_cis_{i}", precompute_freqs_cis(d, max_seq_len, theta),
                                 persistent=False)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return torch.cat([getattr(self, f"freqs_cis_{i}")[ids[..., i]] for i in range(self.n_axes)],
                         dim=-1)


class Timesteps(nn.Module):
    """diffusers Timesteps(num_channels, flip_sin_to_cos=True, downscale_freq_shift=1)."""

    def __init__(self, num_channels: int):
        super().__init__()
        self.num_channels = num_channels

    def forward(self, timesteps: torch.Tensor) -> torch.Tensor:
        half = self.num_channels // 2
        exponent = -math.log(10000) * torch.arange(0, half, dtype=torch.float32)
        exponent = exponent / (half - 1)
        emb = torch.exp(exponent)
        emb = timesteps[:, None].float() * emb[None, :]
        emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
        return torch.cat([emb[:, half:], emb[:, :half]], dim=-1)


class TimestepEmbedding(nn.Module):
    """diffusers TimestepEmbedding(in_channels, time_embed_dim): linear_1 -> SiLU -> linear_2."""

    def __init__(self, in_channels: int, time_embed_dim: int):
        super().__init__()
        self.linear_1 = nn.Linear(in_channels, time_embed_dim)
        self.act = nn.SiLU()
        self.linear_2 = nn.Linear(time_embed_dim, time_embed_dim)

    def forward(self, x):
        return self.linear_2(self.act(self.linear_1(x)))


class TimestepEncoder(nn.Module):
    def __init__(self, embedding_dim: int):
        super().__init__()
        self.time_proj = Timesteps(256)
        self.timestep_embedder = TimestepEmbedding(256, embedding_dim)

    def forward(self, timesteps):
        dtype = next(self.parameters()).dtype
        return self.timestep_embedder(self.time_proj(timesteps).to(dtype))


class SwiGLUFFN(nn.Module):
    def __init__(self, in_features: int, hidden_features: int):
        super().__init__()
        self.w12 = nn.Linear(in_features, 2 * hidden_features)
        self.w3 = nn.Linear(hidden_features, in_features)

    def forward(self, x):
        x1, x2 = self.w12(x).chunk(2, dim=-1)
        return self.w3(F.silu(x1) * x2)


def _key_mask(parts, dtype):
    """Additive SDPA mask over the concatenated key segments: -inf where a key is masked (0)."""
    kv = torch.cat(parts, dim=1)[:, None, None, :]
    return torch.where(kv == 0, torch.tensor(float("-inf"), dtype=dtype), torch.tensor(0.0, dtype=dtype))


def _split_heads(x, h):
    B, N, D = x.shape
    return x.view(B, N, h, D // h).permute(0, 2, 1, 3).contiguous()


def _merge_heads(x):
    B, H, N, Dh = x.shape
    return x.permute(0, 2, 1, 3).contiguous().view(B, N, H * Dh)


# ----------------------------------------------------------------------------------------------
# MSAT
# ----------------------------------------------------------------------------------------------
class ExpandedDoubleStreamBlock(nn.Module):
    """3-way joint block [VL | SA | P]; identity modulation (temb_type='input_token')."""

    streams = ("sa", "vl", "p")

    def __init__(self, dim: int, heads: int, head_dim: int, mlp_hidden: int, vl_mlp_hidden: int,
                 vl_dim: Optional[int] = None):
        super().__init__()
        self.num_heads = heads
        inner = heads * head_dim
        vl_dim = vl_dim if vl_dim is not None else dim
        widths = {"sa": (dim, mlp_hidden), "vl": (vl_dim, vl_mlp_hidden), "p": (dim, mlp_hidden)}
        for s in self.streams:
            w, hid = widths[s]
            setattr(self, f"{s}_norm1", _ln(w))
            setattr(self, f"{s}_norm2_attn", nn.Identity())
            setattr(self, f"{s}_norm2_mlp", _ln(w))
            setattr(self, f"{s}_norm3_mlp", nn.Identity())
            setattr(self, f"{s}_qkv", nn.Linear(w, 3 * inner))
            setattr(self, f"{s}_proj", nn.Linear(inner, w))
            setattr(self, f"{s}_mlp", SwiGLUFFN(w, hid))
        for s in self.streams:
            setattr(self, f"q_norm_{s}", RMSNorm(head_dim))
            setattr(self, f"k_norm_{s}", RMSNorm(head_dim))

    def forward(self, sa, vl, p, pe, attn_mask=None):
        H = self.num_heads
        qs, ks, vs = [], [], []
        for s, x in (("vl", vl), ("sa", sa), ("p", p)):
            y = getattr(self, f"{s}_norm1")(x)
            q, k, v = [_split_heads(t, H) for t in getattr(self, f"{s}_qkv")(y).chunk(3, dim=-1)]
            B, _, N, Dh = q.shape
            q = getattr(self, f"q_norm_{s}")(q.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
            k = getattr(self, f"k_norm_{s}")(k.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
            qs.append(q)
            ks.append(k)
            vs.append(v)
        q, k, v = torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2)
        if pe is not None:
            q, k = apply_rotary_emb(q, k, pe)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
        n_vl, n_sa = vl.shape[1], sa.shape[1]
        outs = {"vl": _merge_heads(o[:, :, :n_vl]), "sa": _merge_heads(o[:, :, n_vl:n_vl + n_sa]),
                "p": _merge_heads(o[:, :, n_vl + n_sa:])}
        res = {}
        for s, x in (("sa", sa), ("vl", vl), ("p", p)):
            x = x + getattr(self, f"{s}_proj")(outs[s])
            x = x + getattr(self, f"{s}_mlp")(getattr(self, f"{s}_norm2_mlp")(x))
            res[s] = x
        return res["sa"], res["vl"], res["p"]


class DoubleStreamBlock(ExpandedDoubleStreamBlock):
    """2-way joint block [VL | SA] (blocks.py:257-609); same per-stream structure."""

    streams = ("sa", "vl")

    def forward(self, sa, vl, pe, attn_mask=None):
        H = self.num_heads
        qs, ks, vs = [], [], []
        for s, x in (("vl", vl), ("sa", sa)):
            y = getattr(self, f"{s}_norm1")(x)
            q, k, v = [_split_heads(t, H) for t in getattr(self, f"{s}_qkv")(y).chunk(3, dim=-1)]
            B, _, N, Dh = q.shape
            q = getattr(self, f"q_norm_{s}")(q.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
            k = getattr(self, f"k_norm_{s}")(k.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
            qs.append(q)
            ks.append(k)
            vs.append(v)
        q, k, v = torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2)
        if pe is not None:
            q, k = apply_rotary_emb(q, k, pe)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
        n_vl = vl.shape[1]
        outs = {"vl": _merge_heads(o[:, :, :n_vl]), "sa": _merge_heads(o[:, :, n_vl:])}
        res = {}
        for s, x in (("sa", sa), ("vl", vl)):
            x = x + getattr(self, f"{s}_proj")(outs[s])
            x = x + getattr(self, f"{s}_mlp")(getattr(self, f"{s}_norm2_mlp")(x))
            res[s] = x
        return res["sa"], res["vl"]


class SingleStreamBlock(nn.Module):
    """Flux-style single block over [VL_proj | time | SA] (blocks.py:42-254) with SwiGLU,
    RMS QK-norm, LayerNorm pre-norm, no post-norm and identity modulation (input_token):
    x + linear2(cat[attn, mlp_proj(silu(x1) * x2)]) with linear1 = [qkv | x1 | x2]."""

    prefixes = ("",)

    def __init__(self, dim: int, heads: int, head_dim: int, mlp_ratio: float):
        super().__init__()
        self.num_heads = heads
        self.inner_dim = heads * head_dim
        self.expanded = int(dim * mlp_ratio)
        self.mlp_hidden = int(2 / 3 * self.expanded)
        for pre in self.prefixes:
            setattr(self, f"{pre}linear1", nn.Linear(dim, 3 * self.inner_dim + 2 * self.expanded))
            setattr(self, f"{pre}linear2", nn.Linear(self.inner_dim + self.mlp_hidden, dim))
            setattr(self, f"{pre}mlp_proj", nn.Linear(self.expanded, self.mlp_hidden))
            setattr(self, f"{pre}q_norm", RMSNorm(head_dim))
            setattr(self, f"{pre}k_norm", RMSNorm(head_dim))
            setattr(self, f"{pre}pre_norm", _ln(dim))
            setattr(self, f"{pre}post_norm", nn.Identity())

    def _in(self, pre, x):
        H = self.num_heads
        y = getattr(self, f"{pre}pre_norm")(x)
        qkv, mlp = torch.split(getattr(self, f"{pre}linear1")(y), [3 * self.inner_dim, 2 * self.expanded], dim=-1)
        q, k, v = [_split_heads(t, H) for t in qkv.chunk(3, dim=-1)]
        B, _, N, Dh = q.shape
        q = getattr(self, f"{pre}q_norm")(q.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
        k = getattr(self, f"{pre}k_norm")(k.reshape(B * H, N, Dh)).reshape(B, H, N, Dh)
        return q, k, v, mlp

    def _out(self, pre, x, attn, mlp):
        x1, x2 = mlp.chunk(2, dim=-1)
        m = getattr(self, f"{pre}mlp_proj")(F.silu(x1) * x2)
        o = getattr(self, f"{pre}linear2")(torch.cat([attn, m], dim=-1))
        return x + getattr(self, f"{pre}post_norm")(o)

    def forward(self, x, pe, attn_mask=None):
        q, k, v, mlp = self._in("", x)
        if pe is not None:
            q, k = apply_rotary_emb(q, k, pe)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
        return self._out("", x, _merge_heads(o), mlp)


class ExpandedSingleStreamBlock(SingleStreamBlock):
    """Single block with the physics stream beside it: joint attention [VL_proj + SA | P], the
    P stream with its own p_* weights (blocks.py:894-1089)."""

    prefixes = ("", "p_")

    def forward(self, x, pe, attn_mask=None, p=None):
        xq, xk, xv, xm = self._in("", x)
        pq, pk, pv, pm = self._in("p_", p)
        q, k, v = torch.cat([xq, pq], 2), torch.cat([xk, pk], 2), torch.cat([xv, pv], 2)
        if pe is not None:
            q, k = apply_rotary_emb(q, k, pe)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
        n_x = x.shape[1]
        return (self._out("", x, _merge_heads(o[:, :, :n_x]), xm),
                self._out("p_", p, _merge_heads(o[:, :, n_x:]), pm))


class MSAT(nn.Module):
    """MSAT: physics path (ExpandedDoubleStreamBlocks [VL | SA | P], then ExpandedSingleStream
    blocks) or standard path (DoubleStreamBlocks [VL | SA], then SingleStreamBlocks)."""

    def __init__(self, cfg: MsatHeadConfig):
        super().__init__()
        inner = cfg.heads * cfg.head_dim
        assert inner == cfg.dim, "time token projection is the identity only when inner == sa_dim"
        self.cfg = cfg
        self.num_temb_tokens = 1
        self.inner_dim = inner
        self.sa_dim = self.vl_dim = cfg.dim
        self.attention_head_dim = cfg.head_dim
        self.positional_embeddings = cfg.positional_embeddings
        self.use_physics = True
        self.timestep_encoder = TimestepEncoder(inner)
        self.time_token_proj = nn.Identity()
        hd = cfg.head_dim
        if cfg.positional_embeddings == "rope_sa_only":
            axes = [hd // 4, hd - hd // 4]
        elif cfg.positional_embeddings == "rope_vl_sa":
            axes = [hd - hd // 4, hd // 4]
        else:
            raise ValueError(cfg.positional_embeddings)
        self.rope_embedder = RoPEEmbedder1D(hd, axes, cfg.rope_theta, cfg.max_seq_len)
        self.use_physics = cfg.use_physics
        self.vl_dim = cfg.vl_width
        self.vl_proj_to_sa = (nn.Linear(cfg.vl_width, cfg.dim) if cfg.vl_width != cfg.dim
                              else nn.Identity())
        dbl = ExpandedDoubleStreamBlock if cfg.use_physics else DoubleStreamBlock
        self.double_blocks = nn.ModuleList(
            dbl(cfg.dim, cfg.heads, hd, cfg.mlp_hidden, cfg.vl_mlp_hidden, cfg.vl_width)
            for _ in range(cfg.depth))
        sgl = ExpandedSingleStreamBlock if cfg.use_physics else SingleStreamBlock
        self.single_blocks = nn.ModuleList(
            sgl(cfg.dim, cfg.heads, hd, cfg.mlp_ratio) for _ in range(cfg.depth_single))
        if cfg.use_physics:
            self.norm_out_physics = _ln(cfg.dim)
            self.proj_out_physics_1 = nn.Linear(inner, 2 * cfg.dim)
            self.proj_out_physics_2 = nn.Linear(cfg.dim, cfg.out_dim)
        self.norm_out = _ln(cfg.dim)
        self.proj_out_1 = nn.Linear(inner, 2 * cfg.dim)
        self.proj_out_2 = nn.Linear(cfg.dim, cfg.out_dim)

    def position_ids(self, B: int, n_vl: int, n_sa: int, n_p: int) -> torch.Tensor:
        """Position ids over [VL | SA(time, state, actions) | P] (msat.py:583-631)."""
        ids = torch.zeros(B, n_vl + n_sa + n_p, 2, dtype=torch.long)
        sa0, p0 = n_vl, n_vl + n_sa
        if self.cfg.positional_embeddings == "rope_vl_sa":
            ids[:, :n_vl, 0] = torch.arange(n_vl)
            start = 2
        else:
            start = 1
        ids[:, sa0, 1] = 0
        ids[:, sa0 + 1:p0, 1] = torch.arange(start, start + n_sa - 1)
        ids[:, p0:, 0] = 1
        ids[:, p0:, 1] = torch.arange(n_p)
        return ids

    def position_ids_standard(self, B: int, n_vl: int, n_sa: int) -> torch.Tensor:
        """Position ids of the double blocks over [VL | SA(time, state, actions)]
        (msat.py:369-420): time (0, 0), S/A (0, 1..) — rope_vl_sa: VL (j, 0), S/A (0, 2..)."""
        ids = torch.zeros(B, n_vl + n_sa, 2, dtype=torch.long)
        if self.cfg.positional_embeddings == "rope_vl_sa":
            ids[:, :n_vl, 0] = torch.arange(n_vl)
            start = 2
        else:
            start = 1
        ids[:, n_vl + 1:, 1] = torch.arange(start, start + n_sa - 1)
        return ids

    def position_ids_single(self, B: int, n_vl: int, n_sa_pure: int, n_p: int = 0) -> torch.Tensor:
        """Position ids of the single blocks over [VL_proj | time | S/A (| P)]
        (msat.py:460-505, 676-709): time (0, 0), S/A (0, 2..) in both RoPE modes, VL (j, 0) under
        rope_vl_sa, P (1, 0..)."""
        n_x = n_vl + 1 + n_sa_pure
        ids = torch.zeros(B, n_x + n_p, 2, dtype=torch.long)
        if self.cfg.positional_embeddings == "rope_vl_sa":
            ids[:, :n_vl, 0] = torch.arange(n_vl)
        ids[:, n_vl + 1:n_x, 1] = torch.arange(2, 2 + n_sa_pure)
        if n_p:
            ids[:, n_x:, 0] = 1
            ids[:, n_x:, 1] = torch.arange(n_p)
        return ids

    def forward_standard(self, hidden_states, encoder_hidden_states, timestep, return_hidden=False,
                         encoder_attention_mask=None):
        """Standard path without physics (msat.py:363-556); a VL key mask as blocks.py:557-576 and
        msat.py:517-531 (VL keys masked, time / S / A keys always visible)."""
        temb = self.timestep_encoder(timestep)
        time_token = self.time_token_proj(temb).unsqueeze(1)
        sa = torch.cat([time_token, hidden_states], dim=1)
        vl = encoder_hidden_states
        B = sa.shape[0]
        pe = self.rope_embedder(self.position_ids_standard(B, vl.shape[1], sa.shape[1]))
        mask = None
        if encoder_attention_mask is not None:
            vm = encoder_attention_mask
            mask = _key_mask([vm, torch.ones(B, sa.shape[1], dtype=vm.dtype)], sa.dtype)
        hidden = []
        for blk in self.double_blocks:
            sa, vl = blk(sa, vl, pe, mask)
            if return_hidden:
                hidden.append((sa, vl))
        time_token, sa = sa[:, :self.num_temb_tokens], sa[:, self.num_temb_tokens:]
        if len(self.single_blocks):
            x = torch.cat([self.vl_proj_to_sa(vl), time_token, sa], dim=1)
            pe_s = self.rope_embedder(self.position_ids_single(B, vl.shape[1], sa.shape[1]))
            mask_s = None
            if encoder_attention_mask is not None:
                vm = encoder_attention_mask
                mask_s = _key_mask([vm, torch.ones(B, x.shape[1] - vl.shape[1], dtype=vm.dtype)], x.dtype)
            for blk in self.single_blocks:
                x = blk(x, pe_s, mask_s)
                if return_hidden:
                    hidden.append((x,))
            sa = x[:, -sa.shape[1]:]
        shift, scale = self.proj_out_1(F.silu(temb)).chunk(2, dim=1)
        a = self.proj_out_2(self.norm_out(sa) * (1 + scale[:, None]) + shift[:, None])
        out = {"action": a}
        return (out, hidden) if return_hidden else out

    def forward(self, hidden_states, encoder_hidden_states, timestep, physics_embs=None,
                encoder_attention_mask=None, physics_attention_mask=None, return_hidden=False):
        if not self.use_physics:
            return self.forward_standard(hidden_states, encoder_hidden_states, timestep, return_hidden,
                                         encoder_attention_mask)
        temb = self.timestep_encoder(timestep)
        time_token = self.time_token_proj(temb).unsqueeze(1)
        sa = torch.cat([time_token, hidden_states], dim=1)
        vl, p = encoder_hidden_states, physics_embs
        B = sa.shape[0]
        pe = self.rope_embedder(self.position_ids(B, vl.shape[1], sa.shape[1], p.shape[1]))
        attn_mask = None
        if encoder_attention_mask is not None or physics_attention_mask is not None:
            vm = encoder_attention_mask if encoder_attention_mask is not None else \
                torch.ones(B, vl.shape[1], dtype=sa.dtype)
            sm = torch.ones(B, sa.shape[1], dtype=vm.dtype)
            pm = (physics_attention_mask[:, None].expand(-1, p.shape[1]).to(vm.dtype)
                  if physics_attention_mask is not None else torch.ones(B, p.shape[1], dtype=vm.dtype))
            kv = torch.cat([vm, sm, pm], dim=1)[:, None, None, :]
            attn_mask = torch.where(kv == 0, torch.tensor(float("-inf"), dtype=sa.dtype),
                                    torch.tensor(0.0, dtype=sa.dtype))
        hidden = []
        for blk in self.double_blocks:
            sa, vl, p = blk(sa, vl, p, pe, attn_mask)
            if return_hidden:
                hidden.append((sa, vl, p))
        time_token, sa = sa[:, :self.num_temb_tokens], sa[:, self.num_temb_tokens:]
        if len(self.single_blocks):
            x = torch.cat([self.vl_proj_to_sa(vl), time_token, sa], dim=1)
            pe_s = self.rope_embedder(self.position_ids_single(B, vl.shape[1], sa.shape[1], p.shape[1]))
            mask_s = None  # [VL_proj + time + S/A | P] (msat.py:716-745)
            if encoder_attention_mask is not None or physics_attention_mask is not None:
                if encoder_attention_mask is not None:
                    vm = encoder_attention_mask
                    xm = torch.cat([vm, torch.ones(B, x.shape[1] - vl.shape[1], dtype=vm.dtype)], dim=1)
                else:
                    xm = torch.ones(B, x.shape[1], dtype=x.dtype)
                pm = (physics_attention_mask[:, None].expand(-1, p.shape[1]).to(xm.dtype)
                      if physics_attention_mask is not None else torch.ones(B, p.shape[1], dtype=xm.dtype))
                mask_s = _key_mask([xm, pm], x.dtype)
            for blk in self.single_blocks:
                x, p = blk(x, pe_s, mask_s, p)
                if return_hidden:
                    hidden.append((x, p))
            sa = x[:, -sa.shape[1]:]
        shift, scale = self.proj_out_1(F.silu(temb)).chunk(2, dim=1)
        a = self.proj_out_2(self.norm_out(sa) * (1 + scale[:, None]) + shift[:, None])
        pshift, pscale = self.proj_out_physics_1(F.silu(temb)).chunk(2, dim=1)
        ph = self.proj_out_physics_2(self.norm_out_physics(p) * (1 + pscale[:, None]) + pshift[:, None])
        out = {"action": a, "physics": ph}
        return (out, hidden) if return_hidden else out


# ----------------------------------------------------------------------------------------------
# encoders / decoders
# ----------------------------------------------------------------------------------------------
class SinusoidalPositionalEncoding(nn.Module):
    def __init__(self, embedding_dim: int):
        super().__init__()
        self.embedding_dim = embedding_dim

    def forward(self, timesteps):
        timesteps = timesteps.float()
        half = self.embedding_dim // 2
        exponent = -torch.arange(half, dtype=torch.float) * (torch.log(torch.tensor(10000.0)) / half)
        freqs = timesteps.unsqueeze(-1) * exponent.exp()
        return torch.cat([torch.sin(freqs), torch.cos(freqs)], dim=-1)


class CategorySpecificLinear(nn.Module):
    def __init__(self, num_categories: int, input_dim: int, hidden_dim: int):
        super().__init__()
        self.W = nn.Parameter(0.02 * torch.randn(num_categories, input_dim, hidden_dim))
        self.b = nn.Parameter(torch.zeros(num_categories, hidden_dim))

    def forward(self, x, cat_ids):
        return torch.bmm(x, self.W[cat_ids]) + self.b[cat_ids].unsqueeze(1)


class CategorySpecificMLP(nn.Module):
    def __init__(self, num_categories, input_dim, hidden_dim, output_dim):
        super().__init__()
        self.layer1 = CategorySpecificLinear(num_categories, input_dim, hidden_dim)
        self.layer2 = CategorySpecificLinear(num_categories, hidden_dim, output_dim)

    def forward(self, x, cat_ids):
        return self.layer2(F.relu(self.layer1(x, cat_ids)), cat_ids)


class MultiEmbodimentActionEncoder(nn.Module):
    def __init__(self, action_dim, hidden_size, num_embodiments):
        super().__init__()
        self.W1 = CategorySpecificLinear(num_embodiments, action_dim, hidden_size)
        self.W2 = CategorySpecificLinear(num_embodiments, 2 * hidden_size, hidden_size)
        self.W3 = CategorySpecificLinear(num_embodiments, hidden_size, hidden_size)
        self.pos_encoding = SinusoidalPositionalEncoding(hidden_size)

    def forward(self, actions, timesteps, cat_ids):
        B, T, _ = actions.shape
        if timesteps.dim() == 1:
            timesteps = timesteps.unsqueeze(1).expand(-1, T)
        a = self.W1(actions, cat_ids)
        tau = self.pos_encoding(timesteps).to(dtype=a.dtype)
        x = self.W2(torch.cat([a, tau], dim=-1), cat_ids)
        x = x * torch.sigmoid(x)
        return self.W3(x, cat_ids)


class PhysicalSignalEncoder(nn.Module):
    def __init__(self, input_dim, hidden_dim, output_dim):
        super().__init__()
        self.W1 = nn.Linear(input_dim, hidden_dim)
        self.W2 = nn.Linear(2 * hidden_dim, hidden_dim)
        self.W3 = nn.Linear(hidden_dim, output_dim)
        self.pos_encoding = SinusoidalPositionalEncoding(hidden_dim)

    def forward(self, x):
        B, T, _ = x.shape
        h = self.W1(x)
        pos = self.pos_encoding(torch.arange(T).float().unsqueeze(0).expand(B, -1)).to(h.dtype)
        return self.W3(F.silu(self.W2(torch.cat([h, pos], dim=-1))))


class PhysicsNoiseEncoder(PhysicalSignalEncoder):
    def forward(self, x, timesteps):
        B, T, _ = x.shape
        t = timesteps.unsqueeze(1).expand(-1, T)
        h = self.W1(x)
        temb = self.pos_encoding(t).to(h.dtype)
        return self.W3(F.silu(self.W2(torch.cat([h, temb], dim=-1))))


class PhysicalSignalDecoder(nn.Module):
    def __init__(self, input_dim, hidden_dim, output_dim):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(input_dim, hidden_dim), nn.SiLU(),
                                 nn.Linear(hidden_dim, output_dim))

    def forward(self, x):
        return self.net(x)


class PhysicsHead(nn.Module):
    def __init__(self, physics_dim, embed_dim, msat_output_dim, hist_len, fut_len):
        super().__init__()
        self.physics_dim = physics_dim
        self.physics_hist_len = hist_len
        self.physics_fut_len = fut_len
        self.physics_cond_encoder = PhysicalSignalEncoder(physics_dim, embed_dim, embed_dim)
        self.physics_fut_encoder = PhysicsNoiseEncoder(physics_dim, embed_dim, embed_dim)
        self.physics_decoder = PhysicalSignalDecoder(msat_output_dim, embed_dim, physics_dim)


class ActionHead(nn.Module):
    """RLDXActionModel's inference sub-modules with the reference attribute names."""

    def __init__(self, cfg: MsatHeadConfig):
        super().__init__()
        self.cfg = cfg
        self.model = MSAT(cfg)
        self.state_encoder = CategorySpecificMLP(cfg.num_embodiments, cfg.state_dim, cfg.dec_hidden, cfg.dim)
        self.action_encoder = MultiEmbodimentActionEncoder(cfg.action_dim, cfg.dim, cfg.num_embodiments)
        self.action_decoder = CategorySpecificMLP(cfg.num_embodiments, cfg.out_dim, cfg.dec_hidden, cfg.action_dim)
        self.position_embedding = nn.Embedding(cfg.pos_emb_len, cfg.dim)
        self.vlln = nn.Identity()
        if cfg.use_physics:
            self.physics = PhysicsHead(cfg.physics_dim, cfg.dim, cfg.out_dim, cfg.physics_hist,
                                       cfg.physics_fut)
        self.use_physics = cfg.use_physics
        self.action_horizon = cfg.horizon
        self.action_dim = cfg.action_dim
        self.num_inference_timesteps = cfg.num_steps


def init_weights(module: nn.Module, seed: int, std: float = 0.02) -> nn.Module:
    """Seeded random init: every parameter ~ N(0, std) except RMSNorm scales ~ 1 + N(0, std)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
            noise = torch.randn(p.shape, generator=g, dtype=torch.float32) * std
            if name.endswith(("norm_sa.weight", "norm_vl.weight", "norm_p.weight",
                              "q_norm.weight", "k_norm.weight")):
                noise = noise + 1.0
            p.copy_(noise.to(p.dtype))
    return module


@torch.no_grad()
def denoise(head: nn.Module, vl_embs, state, embodiment_id, init_noise, physics_hist=None,
            physics_noise=None, num_steps: int = 4, return_trace: bool = False, prefix_actions=None,
            vl_mask=None, physics_mask=None):
    """Control step with vanilla_action_head_forward semantics (benchmark_action_model.py:50-123).

    prefix_actions (B, d, action_dim): RTC trained-mode inpainting as GraphSafeActionModel.forward
    (graph_safe_action_model.py:196-300): the first d action tokens are locked to the prefix
    before every action encoding and after every Euler update, and their encoder time is 1.0
    while the others use the step's t.

    vl_mask (B, n_vl) / physics_mask (B,): key masks (1 = visible) of the backbone tokens and of
    each observation's physics tokens, as get_action_with_features passes them to MSAT
    (rldx/model/core/rldx.py:619-621, 660-666; physics_head.py:232-244); an all-ones VL mask is
    dropped like the reference does."""
    if vl_mask is not None and bool(vl_mask.all()):
        vl_mask = None
    msat = head.model
    dt = 1.0 / num_steps
    vl = head.vlln(vl_embs)
    B = vl.shape[0]
    horizon = init_noise.shape[1]
    d = 0 if prefix_actions is None else prefix_actions.shape[1]
    state_features = head.state_encoder(state, embodiment_id)
    pos_embs = head.position_embedding(torch.arange(horizon)).unsqueeze(0)
    current = init_noise.clone()
    if d:
        current[:, :d] = prefix_actions

    def encode(t):
        timesteps = torch.tensor([t / float(num_steps)], dtype=vl.dtype).expand(B)
        t_enc = timesteps
        if d:
            t_enc = timesteps.unsqueeze(1).expand(-1, horizon).clone()
            t_enc[:, :d] = 1.0
            current[:, :d] = prefix_actions
        af = head.action_encoder(current, t_enc, embodiment_id) + pos_embs
        return timesteps, torch.cat([state_features, af], dim=1)

    def euler(cur, out):
        pred = head.action_decoder(out["action"], embodiment_id)[:, -horizon:]
        cur = cur + dt * pred
        if d:
            cur[:, :d] = prefix_actions
        return cur

    if not head.use_physics:
        trace = []
        for t in range(num_steps):
            timesteps, sa = encode(t)
            out, hidden = msat(sa, vl, timesteps, encoder_attention_mask=vl_mask, return_hidden=True)
            current = euler(current, out)
            if return_trace:
                trace.append({"hidden": hidden, "out": out, "actions": current})
        return (current, trace) if return_trace else current
    phys = head.physics
    physics_hist_tok = phys.physics_cond_encoder(physics_hist)
    physics_fut = physics_noise.clone()
    trace = []
    for t in range(num_steps):
        timesteps, sa = encode(t)
        pe = torch.cat([physics_hist_tok, phys.physics_fut_encoder(physics_fut, timesteps)], dim=1)
        out, hidden = msat(sa, vl, timesteps, pe, encoder_attention_mask=vl_mask,
                           physics_attention_mask=physics_mask, return_hidden=True)
        current = euler(current, out)
        physics_fut = physics_fut + dt * phys.physics_decoder(out["physics"][:, -phys.physics_fut_len:])
        if return_trace:
            trace.append({"hidden": hidden, "out": out, "actions": current, "physics_fut": physics_fut})
    return (current, trace) if return_trace else current


def make_inputs(cfg: MsatHeadConfig, batch: int, seed: int = 42, dtype=torch.float32,
                emb_ids: Optional[list] = None):
    """Seeded synthetic inputs with the shapes of BASELINE config 2 (vl ~ N(0,1), state * 0.01,
    physics ~ N(0,1), init noise ~ N(0,1) from seed + 1, like benchmark_action_model.py:225-241)."""
    g = torch.Generator().manual_seed(seed)
    vl = torch.randn(batch, cfg.n_vl, cfg.vl_width, generator=g)
    state = torch.randn(batch, cfg.n_state, cfg.state_dim, generator=g) * 0.01
    physics_hist = torch.randn(batch, cfg.physics_hist, cfg.physics_dim, generator=g)
    g2 = torch.Generator().manual_seed(seed + 1)
    init_noise = torch.randn(batch, cfg.horizon, cfg.action_dim, generator=g2)
    physics_noise = torch.randn(batch, cfg.physics_fut, cfg.physics_dim, generator=g2)
    ids = torch.tensor(emb_ids if emb_ids is not None else [0] * batch, dtype=torch.long)
    cast = lambda t: t.to(dtype)  # noqa: E731
    return {"vl": cast(vl), "state": cast(state), "embodiment_id": ids,
            "init_noise": cast(init_noise), "physics_hist": cast(physics_hist),
            "physics_noise": cast(physics_noise)}
