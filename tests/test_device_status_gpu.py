"""Device-error reporting of the runtimes, tested the way this pool allows: a bounded wait on a
barrier that nothing arrives on runs out (the self-test kernel), records its code and returns;
the GPU context stays usable.  The control step then reports that code -- synchronously from
rldx_msat_step_host, and through the handle's status after the asynchronous rldx_msat_step --
while its own kernels run from a clean error word and still compute the right actions.  This
replaces the reference's silent fall-back to the vanilla path on a failure
(rldx/inference/serve_optimization.py:432-516)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from oracle import msat_oracle as om  # noqa: E402
from rldx_b200 import _lib, ops  # noqa: E402
from rldx_b200.chain import B200ExpandedActionHeadChain  # noqa: E402

BF = torch.bfloat16
SELFTEST = 0x400
LIMIT = 2_000_000  # SM cycles: about a millisecond


@pytest.fixture(scope="module")
def small_chain(cuda):
    cfg = om.MsatHeadConfig(n_vl=64, horizon=16, physics_hist=16, physics_fut=16, dim=256, heads=4,
                            depth=2, mlp_ratio=3.0, out_dim=128, action_dim=32, state_dim=64,
                            dec_hidden=128, physics_dim=37, num_embodiments=4)
    head = om.init_weights(om.ActionHead(cfg), seed=0).to(BF)
    inp = om.make_inputs(cfg, batch=2, seed=1, dtype=BF, emb_ids=[0, 3])
    chain = B200ExpandedActionHeadChain(head, cuda)
    d = {k: v.to(cuda) for k, v in inp.items()}
    args = (d["vl"], d["state"], d["embodiment_id"], d["init_noise"], d["physics_hist"], d["physics_noise"])
    ref = chain(*args).cpu()
    torch.cuda.synchronize()
    assert chain.device_status() == 0
    host = {k: v.contiguous().pin_memory() for k, v in inp.items()}
    return chain, args, host, ref


def test_wait_selftest_records_its_code(cuda):
    assert ops.device_error() == 0
    ops.wait_selftest(LIMIT)
    assert ops.device_error() == SELFTEST  # synchronizes, reads and clears
    assert ops.device_error() == 0


def test_step_host_reports_an_error_left_by_earlier_work(small_chain):
    chain, _, host, ref = small_chain
    out = torch.empty(ref.shape, dtype=BF).pin_memory()
    ops.wait_selftest(LIMIT)
    with pytest.raises(_lib.RldxError, match="0x400") as e:
        chain.forward_host(host, out)
    assert e.value.code == _lib.RLDX_ERR_DEVICE
    assert torch.equal(out, ref)  # the step took the code first and ran clean
    out.zero_()
    chain.forward_host(host, out)  # the status was cleared: the next step succeeds
    assert torch.equal(out, ref)
    assert ops.device_error() == 0


def test_async_step_status_and_next_call(small_chain):
    chain, args, _, ref = small_chain
    ops.wait_selftest(LIMIT)
    out = chain(*args)  # asynchronous: queued behind the self-test on the same stream
    assert chain.device_status(wait=True) == SELFTEST
    assert torch.equal(out.cpu(), ref)
    assert chain.device_status(wait=True) == 0  # reading cleared it
    ops.wait_selftest(LIMIT)
    chain(*args)
    torch.cuda.synchronize()
    # the next call sees the recorded code of the finished step before queueing more work
    with pytest.raises(_lib.RldxError, match="device error 0x400"):
        chain(*args)
    out = chain(*args)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), ref)
    assert chain.device_status(wait=True) == 0


def test_wait_limit_is_a_run_time_value(small_chain):
    chain, args, _, ref = small_chain
    default = ops.get_wait_limit()
    assert default == 4_000_000_000
    try:
        ops.set_wait_limit(200_000_000)  # ~0.1 s: far above a healthy wait
        assert ops.get_wait_limit() == 200_000_000
        out = chain(*args)
        assert chain.device_status(wait=True) == 0
        assert torch.equal(out.cpu(), ref)
    finally:
        ops.set_wait_limit(default)
    with pytest.raises(_lib.RldxError):
        ops.set_wait_limit(10)
