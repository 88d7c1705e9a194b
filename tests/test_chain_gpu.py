"""End-to-end control step on the GPU (native runtime, one CUDA graph) vs the CPU oracle and
the reference's own golden vectors."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200.chain import B200ExpandedActionHeadChain  # noqa: E402
from oracle import msat_oracle as om  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden"
BF = torch.bfloat16


def cos_sim(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def run_chain(head_bf16, inp, cuda, use_graph=True):
    chain = B200ExpandedActionHeadChain(head_bf16, cuda, use_graph=use_graph)
    dev = {k: v.to(cuda) for k, v in inp.items()}
    out = chain(dev["vl"].to(BF), dev["state"].to(BF), dev["embodiment_id"], init_noise=dev["init_noise"].to(BF),
                physics_hist=dev["physics_hist"].to(BF), physics_init_noise=dev["physics_noise"].to(BF))
    torch.cuda.synchronize()
    return chain, out.cpu()


@pytest.mark.parametrize("batch", [1, 2])
def test_small_head_matches_reference_golden(cuda, batch):
    """Actions within 2e-2 (max-abs) of the reference bf16 eager path on the same inputs."""
    fx16 = torch.load(GOLD / f"head_small_b{batch}_bf16.pt", weights_only=False)
    fx32 = torch.load(GOLD / f"head_small_b{batch}_fp32.pt", weights_only=False)
    cfg = om.MsatHeadConfig(**fx16["config"])
    head = om.init_weights(om.ActionHead(cfg), seed=fx16["seed"]).to(BF)
    _, out = run_chain(head, fx32["inputs"], cuda)
    err16 = (out.float() - fx16["actions"].float()).abs().max().item()
    assert err16 <= 2e-2, err16
    assert cos_sim(out.float(), fx32["actions"]) >= 0.999


def test_graph_replay_is_deterministic(cuda):
    cfg = om.MsatHeadConfig(n_vl=40, horizon=16, physics_hist=16, physics_fut=16, dim=256, heads=4,
                            depth=3, mlp_ratio=3.0, out_dim=128, action_dim=32, state_dim=64,
                            dec_hidden=128, physics_dim=37, num_embodiments=4)
    head = om.init_weights(om.ActionHead(cfg), seed=5).to(BF)
    inp = om.make_inputs(cfg, batch=1, seed=3)
    chain, a = run_chain(head, inp, cuda)
    dev = {k: v.to(cuda) for k, v in inp.items()}
    b = chain(dev["vl"].to(BF), dev["state"].to(BF), dev["embodiment_id"], dev["init_noise"].to(BF),
              dev["physics_hist"].to(BF), dev["physics_noise"].to(BF)).cpu()
    assert torch.equal(a, b)
    # eager launch list (no graph) gives the same bits
    _, c = run_chain(head, inp, cuda, use_graph=False)
    assert torch.equal(a, c)


def test_multi_embodiment_batch(cuda):
    cfg = om.MsatHeadConfig(n_vl=64, horizon=16, physics_hist=16, physics_fut=16, dim=256, heads=4,
                            depth=2, mlp_ratio=3.0, out_dim=128, action_dim=32, state_dim=64,
                            dec_hidden=128, physics_dim=37, num_embodiments=6)
    head = om.init_weights(om.ActionHead(cfg), seed=8)
    inp = om.make_inputs(cfg, batch=3, seed=4, emb_ids=[5, 0, 3])
    ref16 = om.denoise(head.to(BF), *[inp[k].to(BF) if inp[k].is_floating_point() else inp[k]
                                      for k in ("vl", "state", "embodiment_id", "init_noise",
                                                "physics_hist", "physics_noise")], cfg.num_steps)
    _, out = run_chain(head.to(BF), inp, cuda)
    assert (out.float() - ref16.float()).abs().max().item() <= 2e-2
