"""Seeded random-init action-head weights laid out like the reference module tree.

The benchmark and smoke paths have no checkpoint (none is shipped and there is no network),
so they bind the B200 chains to this namespace tree: the same attribute names and tensor shapes
as RLDXActionModel's inference sub-modules (rldx/model/core/rldx.py:43-106), bf16 tensors
created directly on the GPU.  Linear / category weights and biases ~ N(0, std), QK-RMSNorm
scales ~ 1 + N(0, std).

Presets: HeadDims() is BASELINE config 2; production() and production_addons() are the
reference's released head without / with add-ons (rldx/configs/model/rldx.py:81-112: 4 double
+ 8 single blocks, 24 x 64 heads, input_embedding_dim 1536, VL width 4096, max action / state
dim 64, hidden_size 1024; 1244.6 M / 1842.6 M MSAT parameters,
rldx/inference/action_model/README.md:11, 30).
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace as NS

import torch
from torch import nn


@dataclass
class HeadDims:
    """full MSAT action decoder, 16 blocks, hidden 1536, 24 x 64 heads."""

    n_vl: int = 512
    n_state: int = 1
    horizon: int = 16
    physics_hist: int = 16
    physics_fut: int = 16
    dim: int = 1536
    heads: int = 24
    depth: int = 16
    mlp_hidden: int = 4096
    vl_mlp_hidden: int = 4096
    out_dim: int = 1024
    action_dim: int = 32
    state_dim: int = 64
    dec_hidden: int = 1024
    physics_dim: int = 37
    num_embodiments: int = 36
    num_steps: int = 4
    rope_theta: float = 10000.0
    rope_max_seq: int = 1024
    pos_emb_len: int = 1024
    use_physics: bool = True
    vl_dim: int = 1536           # VL stream width of the double blocks
    depth_single: int = 0        # single-stream blocks after the double ones
    single_expanded: int = 6144  # int(dim * mlp_ratio)
    single_mlp_hidden: int = 4096

    @property
    def tokens(self) -> int:
        p = self.physics_hist + self.physics_fut if self.use_physics else 0
        return self.n_vl + 1 + self.n_state + self.horizon + p


def production() -> HeadDims:
    """The released no-add-on head: DoubleStreamBlocks [VL 64 x 4096 | SA 18 x 1536] x 4, then
    SingleStreamBlocks x 8; VL SwiGLU hidden int(2/3 * 4 * 4096) = 10922."""
    return HeadDims(n_vl=64, physics_hist=0, physics_fut=0, depth=4, mlp_hidden=4096, vl_mlp_hidden=10922,
                    action_dim=64, state_dim=64, rope_max_seq=512, use_physics=False, vl_dim=4096,
                    depth_single=8)


def production_addons() -> HeadDims:
    """The released all-add-on head: ExpandedDoubleStreamBlocks [VL 80 x 4096 | SA 18 | P 32] x 4,
    then ExpandedSingleStreamBlocks x 8 (physics 16 history + 16 future tokens, 37 channels)."""
    return HeadDims(n_vl=80, depth=4, mlp_hidden=4096, vl_mlp_hidden=10922, action_dim=64, state_dim=64,
                    rope_max_seq=512, use_physics=True, vl_dim=4096, depth_single=8)


PRESETS = {"c2": HeadDims, "production": production, "production_addons": production_addons}


def random_action_head(d: HeadDims, seed: int = 0, device="cuda", std: float = 0.02,
                       cos_only_rope: bool = True) -> NS:
    g = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16

    def rnd(*shape, mean=0.0):
        return (torch.randn(*shape, generator=g, device=device) * std + mean).to(bf)

    def lin(i, o):
        return NS(weight=rnd(o, i), bias=rnd(o))

    def cat(i, o):
        return NS(W=rnd(d.num_embodiments, i, o), b=rnd(d.num_embodiments, o))

    streams = [("sa", d.dim, d.mlp_hidden), ("vl", d.vl_dim, d.vl_mlp_hidden)]
    if d.use_physics:
        streams.append(("p", d.dim, d.mlp_hidden))
    blocks = []
    for _ in range(d.depth):
        b = NS(num_heads=d.heads)
        for s, width, hid in streams:
            setattr(b, f"{s}_qkv", lin(width, 3 * d.dim))
            setattr(b, f"{s}_proj", lin(d.dim, width))
            setattr(b, f"{s}_mlp", NS(w12=lin(width, 2 * hid), w3=lin(hid, width)))
            setattr(b, f"q_norm_{s}", NS(weight=rnd(64, mean=1.0)))
            setattr(b, f"k_norm_{s}", NS(weight=rnd(64, mean=1.0)))
        blocks.append(b)
    singles = []
    for _ in range(d.depth_single):
        sb = NS(num_heads=d.heads)
        for pre in (("", "p_") if d.use_physics else ("",)):
            setattr(sb, f"{pre}linear1", lin(d.dim, 3 * d.dim + 2 * d.single_expanded))
            setattr(sb, f"{pre}linear2", lin(d.dim + d.single_mlp_hidden, d.dim))
            setattr(sb, f"{pre}mlp_proj", lin(d.single_expanded, d.single_mlp_hidden))
            setattr(sb, f"{pre}q_norm", NS(weight=rnd(64, mean=1.0)))
            setattr(sb, f"{pre}k_norm", NS(weight=rnd(64, mean=1.0)))
            setattr(sb, f"{pre}pre_norm", nn.LayerNorm(d.dim, eps=1e-6, elementwise_affine=False))
            setattr(sb, f"{pre}post_norm", nn.Identity())
        singles.append(sb)
    # RoPEEmbedder1D tables (ops.py:11-25, axes [16, 48] under rope_sa_only); a bf16-loaded
    # module keeps only their real part (the cos-only quirk)
    tables = {}
    for i, dim in enumerate((16, 48)):
        inv = 1.0 / (d.rope_theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
        ang = torch.outer(torch.arange(d.rope_max_seq), inv).float()
        t = torch.polar(torch.ones_like(ang), ang)
        tables[f"freqs_cis_{i}"] = (t.real.to(bf) if cos_only_rope else t).to(device)
    msat = NS(
        double_blocks=blocks, single_blocks=singles, temb_type="input_token", use_physics=d.use_physics,
        positional_embeddings="rope_sa_only", time_token_proj=nn.Identity(),
        timestep_encoder=NS(timestep_embedder=NS(linear_1=lin(256, d.dim), linear_2=lin(d.dim, d.dim))),
        rope_embedder=NS(**tables, theta=d.rope_theta),
        vl_proj_to_sa=lin(d.vl_dim, d.dim) if d.vl_dim != d.dim else nn.Identity(),
        proj_out_1=lin(d.dim, 2 * d.dim), proj_out_2=lin(d.dim, d.out_dim))
    if d.use_physics:
        msat.proj_out_physics_1 = lin(d.dim, 2 * d.dim)
        msat.proj_out_physics_2 = lin(d.dim, d.out_dim)

    def enc():
        return NS(W1=lin(d.physics_dim, d.dim), W2=lin(2 * d.dim, d.dim), W3=lin(d.dim, d.dim))

    physics = None
    if d.use_physics:
        physics = NS(physics_cond_encoder=enc(), physics_fut_encoder=enc(),
                     physics_decoder=NS(net=[lin(d.out_dim, d.dim), None, lin(d.dim, d.physics_dim)]),
                     physics_hist_len=d.physics_hist, physics_fut_len=d.physics_fut,
                     physics_dim=d.physics_dim)
    return NS(
        model=msat,
        state_encoder=NS(layer1=cat(d.state_dim, d.dec_hidden), layer2=cat(d.dec_hidden, d.dim)),
        action_encoder=NS(W1=cat(d.action_dim, d.dim), W2=cat(2 * d.dim, d.dim), W3=cat(d.dim, d.dim)),
        action_decoder=NS(layer1=cat(d.out_dim, d.dec_hidden), layer2=cat(d.dec_hidden, d.action_dim)),
        position_embedding=NS(weight=rnd(d.pos_emb_len, d.dim)),
        physics=physics,
        vlln=nn.Identity(), num_inference_timesteps=d.num_steps, action_horizon=d.horizon)


def random_inputs(d: HeadDims, batch: int, seed: int = 42, device="cuda", pin: bool = False) -> dict:
    """BASELINE config 2 inputs: vl ~ N(0,1), state * 0.01, physics ~ N(0,1), noise ~ N(0,1)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    bf = torch.bfloat16
    t = {
        "vl": torch.randn(batch, d.n_vl, d.vl_dim, generator=g).to(bf),
        "state": (torch.randn(batch, d.n_state, d.state_dim, generator=g) * 0.01).to(bf),
        "embodiment_id": torch.zeros(batch, dtype=torch.int64),
        "init_noise": torch.randn(batch, d.horizon, d.action_dim, generator=g).to(bf),
    }
    if d.use_physics:
        t["physics_hist"] = torch.randn(batch, d.physics_hist, d.physics_dim, generator=g).to(bf)
        t["physics_noise"] = torch.randn(batch, d.physics_fut, d.physics_dim, generator=g).to(bf)
    if device == "cpu":
        return {k: (v.pin_memory() if pin else v) for k, v in t.items()}
    return {k: v.to(device) for k, v in t.items()}
