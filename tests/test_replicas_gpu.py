"""ReplicaPool, the single-process data-parallel endpoint: one action-head replica per device,
each device's share of the observations run on its own stream.  Its actions must equal, bit for
bit, those of a chain bound to that share alone (the replicas share nothing).  With one visible
GPU both replicas live on it, which still runs the per-replica streams and the host gather."""

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from oracle import msat_oracle as om  # noqa: E402
from rldx_b200.chain import B200ExpandedActionHeadChain  # noqa: E402
from rldx_b200.replicas import ReplicaPool, shard_bounds  # noqa: E402

NAMES = ("vl", "state", "embodiment_id", "init_noise", "physics_hist", "physics_noise")
KW = {"vl": "vl_embs", "state": "state", "embodiment_id": "embodiment_id", "init_noise": "init_noise",
      "physics_hist": "physics_hist", "physics_noise": "physics_init_noise"}


def test_pool_matches_chains_bound_to_each_share(cuda):
    cfg = om.MsatHeadConfig(n_vl=64, horizon=16, physics_hist=16, physics_fut=16, dim=256, heads=4,
                            depth=2, mlp_ratio=3.0, out_dim=128, action_dim=32, state_dim=64,
                            dec_hidden=128, physics_dim=37, num_embodiments=4)
    head = om.init_weights(om.ActionHead(cfg), seed=3).to(torch.bfloat16)
    inp = om.make_inputs(cfg, batch=5, seed=9, dtype=torch.bfloat16, emb_ids=[0, 3, 1, 2, 3])
    devices = ["cuda:0", "cuda:1"] if torch.cuda.device_count() >= 2 else [cuda, cuda]
    pool = ReplicaPool(lambda d: B200ExpandedActionHeadChain(head, d), devices)
    host = {KW[k]: inp[k].contiguous().pin_memory() for k in NAMES}
    out = pool(**host)
    again = pool(**host)
    assert out.shape == (5, cfg.horizon, cfg.action_dim) and out.device.type == "cpu"
    assert torch.equal(out, again)
    for r in range(len(pool)):
        s, e = shard_bounds(5, len(pool), r)
        ref = B200ExpandedActionHeadChain(head, cuda)(*[inp[k][s:e].to(cuda) for k in NAMES])
        torch.cuda.synchronize()
        assert torch.equal(out[s:e], ref.cpu()), r


def test_pool_rejects_ragged_batches(cuda):
    pool = ReplicaPool(lambda d: None, [cuda])
    with pytest.raises(ValueError, match="disagree"):
        pool(vl_embs=torch.zeros(3, 4), state=torch.zeros(2, 4))
