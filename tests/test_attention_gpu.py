"""tcgen05 joint attention vs a plain PyTorch fp32 softmax attention of the same inputs."""

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200 import ops  # noqa: E402

BF = torch.bfloat16


def run_case(cuda, B, H, segs, mask=False, seed=0, hd=64, tiles=0):
    L = sum(segs)
    Lp = (L + 7) // 8 * 8
    g = torch.Generator(device=cuda).manual_seed(seed)
    q = torch.randn(B, H, L, hd, device=cuda, generator=g).to(BF)
    k = torch.randn(B, H, L, hd, device=cuda, generator=g).to(BF)
    v = torch.randn(B, H, L, hd, device=cuda, generator=g).to(BF)
    vt = torch.zeros(B, H, hd, Lp, dtype=BF, device=cuda)
    vt[..., :L] = v.transpose(-1, -2)
    key_mask = None
    bias = torch.zeros(B, 1, 1, L, device=cuda)
    if mask:
        key_mask = (torch.rand(B, L, device=cuda, generator=g) > 0.3).to(torch.uint8)
        key_mask[:, segs[0]:] = 1  # the action stream is always visible (blocks.py:852)
        bias = torch.where(key_mask.bool(), 0.0, float("-inf"))[:, None, None, :]
    outs = ops.joint_attention(q, k, vt, segs, key_mask=key_mask, tiles_per_cta=tiles)
    torch.cuda.synchronize()
    s = (q.float() @ k.float().transpose(-1, -2)) / hd ** 0.5 + bias
    ref = torch.softmax(s, dim=-1) @ v.float()  # [B, H, L, hd]
    ref = ref.permute(0, 2, 1, 3).reshape(B, L, H * hd)
    off = 0
    for o, n in zip(outs, segs):
        exp = ref[:, off:off + n].reshape(B * n, H * hd)
        err = (o.float() - exp).abs().max().item()
        assert err < 2e-2, f"segment at {off}: max err {err}"
        off += n
    assert ops.device_error() == 0


@pytest.mark.parametrize("segs", [[1], [5], [64], [65], [127, 1], [128], [129], [256, 16, 16],
                                  [512, 18, 32], [1000, 48]])
def test_joint_attention_lengths(cuda, segs):
    run_case(cuda, 1, 2, segs, seed=len(segs) + sum(segs))


@pytest.mark.parametrize("B,H", [(2, 3), (3, 24)])
def test_joint_attention_batched(cuda, B, H):
    run_case(cuda, B, H, [200, 18, 32], seed=B * 100 + H)


def test_joint_attention_key_mask(cuda):
    run_case(cuda, 2, 4, [96, 18, 32], mask=True, seed=7)


# Launches with no more 128-query tiles than SMs split each tile's keys over two softmax
# warpgroups (head_dim 64); larger ones run one warpgroup per tile.  Both forms, with and
# without a key mask:
@pytest.mark.parametrize("B,segs", [(1, [512, 18, 32]), (8, [512, 18, 32]), (2, [1000, 48])])
@pytest.mark.parametrize("mask", [False, True])
def test_joint_attention_column_split_and_single_warpgroup(cuda, B, segs, mask):
    run_case(cuda, B, 24, segs, mask=mask, seed=B * 10 + len(segs) + int(mask))


@pytest.mark.parametrize("segs", [[1], [65], [240, 32, 16], [496, 32, 16], [1008, 32, 16]])
def test_joint_attention_head_dim_128(cuda, segs):
    """head_dim 128 (the joint-attention sweep's shape: segments (L-48):32:16, 16 heads)."""
    run_case(cuda, 2, 16, segs, seed=sum(segs), hd=128)


@pytest.mark.parametrize("segs", [[2032, 32, 16], [4080, 32, 16]])
def test_joint_attention_head_dim_128_long(cuda, segs):
    """The two longest lengths of the joint-attention sweep (L 2080 and 4128, segments
    (L-48):32:16, 16 heads of 128)."""
    run_case(cuda, 1, 16, segs, seed=sum(segs), hd=128)


def test_joint_attention_head_dim_128_key_mask(cuda):
    run_case(cuda, 2, 4, [200, 32, 16], mask=True, seed=3, hd=128)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("segs", [[1], [100, 28], [129], [200, 18, 32], [256], [300, 30, 20], [512, 18, 32]])
def test_joint_attention_two_tiles_per_cta(cuda, hd, segs):
    """Two 128-query tiles per CTA (two softmax warpgroups), including a last CTA whose second
    tile lies wholly past L."""
    run_case(cuda, 2, 3, segs, seed=hd + sum(segs), hd=hd, tiles=2)


def test_joint_attention_two_tiles_key_mask(cuda):
    run_case(cuda, 2, 4, [300, 18, 32], mask=True, seed=5, tiles=2)


def run_gqa_causal(cuda, B, H, Hkv, L, hd, causal, seed=0, tiles=0):
    Lp = (L + 7) // 8 * 8
    g = torch.Generator(device=cuda).manual_seed(seed)
    q = torch.randn(B, H, L, hd, device=cuda, generator=g).to(BF)
    k = torch.randn(B, Hkv, L, hd, device=cuda, generator=g).to(BF)
    v = torch.randn(B, Hkv, L, hd, device=cuda, generator=g).to(BF)
    vt = torch.zeros(B, Hkv, hd, Lp, dtype=BF, device=cuda)
    vt[..., :L] = v.transpose(-1, -2)
    (out,) = ops.attention(q, k, vt, causal=causal, tiles_per_cta=tiles)
    torch.cuda.synchronize()
    rep = H // Hkv
    kf = k.float().repeat_interleave(rep, dim=1)
    vf = v.float().repeat_interleave(rep, dim=1)
    s = (q.float() @ kf.transpose(-1, -2)) / hd ** 0.5
    if causal:
        s = s.masked_fill(torch.ones(L, L, dtype=torch.bool, device=cuda).triu(1), float("-inf"))
    ref = (torch.softmax(s, dim=-1) @ vf).permute(0, 2, 1, 3).reshape(B * L, H * hd)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err
    assert ops.device_error() == 0


@pytest.mark.parametrize("L", [1, 63, 64, 65, 128, 129, 300, 848])
@pytest.mark.parametrize("hd", [64, 128])
def test_causal_gqa_attention(cuda, L, hd):
    """Decoder prefill form: causal mask, 16 query heads over 2 kv heads (Qwen3 GQA)."""
    run_gqa_causal(cuda, 2, 16, 2, L, hd, causal=True, seed=L + hd)


def test_gqa_non_causal_and_two_tiles(cuda):
    run_gqa_causal(cuda, 1, 8, 4, 300, 128, causal=False, seed=1)
    run_gqa_causal(cuda, 2, 16, 2, 520, 128, causal=True, seed=2, tiles=2)
