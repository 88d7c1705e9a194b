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
  ExpandedDoubleStreamBlock    rldx/model/modules/action_model/blocks.py:612-891 (input_token
                               temb => identity modulation, blocks.py:737-760)
  MSAT._forward_physics        rldx/model/modules/action_model/msat.py:558-781 (0 single blocks)
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
    dim: int = 1536  # sa_dim == vl_dim == p_dim == heads * head_dim
    heads: int = 24
    head_dim: int = 64
    depth: int = 16
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
    def vl_mlp_hidden(self) -> int:
        r = self.vl_mlp_ratio if self.vl_mlp_ratio is not None else self.mlp_ratio
        return int(2 / 3 * int(self.dim * r))


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

    def __init__(self, dim: int, heads: int, head_dim: int, mlp_hidden: int, vl_mlp_hidden: int):
        super().__init__()
        self.num_heads = heads
        inner = heads * head_dim
        for s, hid in (("sa", mlp_hidden), ("vl", vl_mlp_hidden), ("p", mlp_hidden)):
            setattr(self, f"{s}_norm1", _ln(dim))
            setattr(self, f"{s}_norm2_attn", nn.Identity())
            setattr(self, f"{s}_norm2_mlp", _ln(dim))
            setattr(self, f"{s}_norm3_mlp", nn.Identity())
            setattr(self, f"{s}_qkv", nn.Linear(dim, 3 * inner))
            setattr(self, f"{s}_proj", nn.Linear(inner, dim))
            setattr(self, f"{s}_mlp", SwiGLUFFN(dim, hid))
        for s in ("sa", "vl", "p"):
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


class MSAT(nn.Module):
    """MSAT with physics stream, `depth` ExpandedDoubleStreamBlocks and no single blocks."""

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
        self.vl_proj_to_sa = nn.Identity()
        self.double_blocks = nn.ModuleList(
            ExpandedDoubleStreamBlock(cfg.dim, cfg.heads, hd, cfg.mlp_hidden, cfg.vl_mlp_hidden)
            for _ in range(cfg.depth))
        self.single_blocks = nn.ModuleList()
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

    def forward(self, hidden_states, encoder_hidden_states, timestep, physics_embs,
                encoder_attention_mask=None, physics_attention_mask=None, return_hidden=False):
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
        sa = sa[:, self.num_temb_tokens:]
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
        self.physics = PhysicsHead(cfg.physics_dim, cfg.dim, cfg.out_dim, cfg.physics_hist, cfg.physics_fut)
        self.use_physics = True
        self.action_horizon = cfg.horizon
        self.action_dim = cfg.action_dim
        self.num_inference_timesteps = cfg.num_steps


def init_weights(module: nn.Module, seed: int, std: float = 0.02) -> nn.Module:
    """Seeded random init: every parameter ~ N(0, std) except RMSNorm scales ~ 1 + N(0, std)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
            noise = torch.randn(p.shape, generator=g, dtype=torch.float32) * std
            if name.endswith("norm_sa.weight") or name.endswith("norm_vl.weight") or \
                    name.endswith("norm_p.weight"):
                noise = noise + 1.0
            p.copy_(noise.to(p.dtype))
    return module


@torch.no_grad()
def denoise(head: nn.Module, vl_embs, state, embodiment_id, init_noise, physics_hist, physics_noise,
            num_steps: int, return_trace: bool = False):
    """Control step with vanilla_action_head_forward semantics (benchmark_action_model.py:50-123)."""
    msat = head.model
    dt = 1.0 / num_steps
    vl = head.vlln(vl_embs)
    B = vl.shape[0]
    horizon = init_noise.shape[1]
    state_features = head.state_encoder(state, embodiment_id)
    pos_embs = head.position_embedding(torch.arange(horizon)).unsqueeze(0)
    current = init_noise.clone()
    phys = head.physics
    physics_hist_tok = phys.physics_cond_encoder(physics_hist)
    physics_fut = physics_noise.clone()
    trace = []
    for t in range(num_steps):
        timesteps = torch.tensor([t / float(num_steps)], dtype=vl.dtype).expand(B)
        af = head.action_encoder(current, timesteps, embodiment_id) + pos_embs
        sa = torch.cat([state_features, af], dim=1)
        pe = torch.cat([physics_hist_tok, phys.physics_fut_encoder(physics_fut, timesteps)], dim=1)
        out, hidden = msat(sa, vl, timesteps, pe, return_hidden=True)
        pred = head.action_decoder(out["action"], embodiment_id)[:, -horizon:]
        current = current + dt * pred
        physics_fut = physics_fut + dt * phys.physics_decoder(out["physics"][:, -phys.physics_fut_len:])
        if return_trace:
            trace.append({"hidden": hidden, "out": out, "actions": current, "physics_fut": physics_fut})
    return (current, trace) if return_trace else current


def make_inputs(cfg: MsatHeadConfig, batch: int, seed: int = 42, dtype=torch.float32,
                emb_ids: Optional[list] = None):
    """Seeded synthetic inputs with the shapes of BASELINE config 2 (vl ~ N(0,1), state * 0.01,
    physics ~ N(0,1), init noise ~ N(0,1) from seed + 1, like benchmark_action_model.py:225-241)."""
    g = torch.Generator().manual_seed(seed)
    vl = torch.randn(batch, cfg.n_vl, cfg.dim, generator=g)
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
