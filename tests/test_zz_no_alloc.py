"""rldx_gemm_static_ws, the GEMM entry point that allocates nothing (its K-split workspace is
a static device array of the library), checked through the C ABI against rldx_gemm_ws, the
entry point that takes a caller workspace, on two calls in a row.

The file name makes pytest collect it last, so a run that stops at the first failure has run
every other test before this one; it must pass alone in a fresh process and after the rest."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

import rldx_b200  # noqa: E402,F401
from rldx_b200 import _lib, ops  # noqa: E402

BF = torch.bfloat16
STATIC_SCRATCH_BYTES = 8 << 20


def _static(descs):
    arr = (_lib.GemmDesc * len(descs))(*descs)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.load().rldx_gemm_static_ws(arr, len(descs), stream))


def _problems(cuda, seed):
    """A w3-like projection of the 18 action-stream rows (K = 4096 -> 1536) with a residual add:
    its few output tiles leave most SMs idle, so the planner splits it along K, and any split
    plan of one 18-row problem needs less workspace than the static scratch holds."""
    g = torch.Generator(device=cuda).manual_seed(seed)
    keep, descs, outs = [], [], []
    for M in (18,):
        x = torch.randn(M, 4096, device=cuda, generator=g).to(BF)
        w = (torch.randn(1536, 4096, device=cuda, generator=g) * 0.03).to(BF)
        b = (torch.randn(1536, device=cuda, generator=g) * 0.1).to(BF)
        res = torch.randn(M, 1536, device=cuda, generator=g).to(BF)
        out = torch.empty(M, 1536, dtype=BF, device=cuda)
        keep += [x, w, b, res, out]  # descriptors hold raw pointers: keep the tensors alive
        descs.append(ops.gemm_desc(x, w, out, b, add=res))
        outs.append(out)
    return keep, descs, outs


def test_static_scratch_matches_caller_workspace(cuda):
    keep, descs, outs = _problems(cuda, 77)
    need = ops.gemm_workspace_size(descs)
    assert 0 < need <= STATIC_SCRATCH_BYTES, need
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    for _ in range(2):  # two calls in a row of each entry point
        ops.gemm(descs, workspace=ws)
        torch.cuda.synchronize()
        want = [o.clone() for o in outs]
        for o in outs:
            o.zero_()
        _static(descs)
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            # same plan, same split order: the results agree bit for bit
            assert torch.equal(o, w)
    assert ops.device_error() == 0


def test_static_scratch_call_allocates_no_device_memory(cuda):
    """A warm call leaves the device's free memory where it was: the K-split partials and
    counters live in the library's static array, and nothing else is allocated."""
    keep, descs, outs = _problems(cuda, 78)
    _static(descs)  # first call on this device: looks the scratch address up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _static(descs)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert ops.device_error() == 0


def test_static_scratch_rejects_plans_that_do_not_fit(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(512, 8192, device=cuda, generator=g).to(BF)
    w = (torch.randn(1024, 8192, device=cuda, generator=g) * 0.02).to(BF)
    out = torch.zeros(512, 1024, dtype=BF, device=cuda)
    descs = [ops.gemm_desc(x, w, out, tile_n=256)]
    assert ops.gemm_workspace_size(descs) > STATIC_SCRATCH_BYTES
    with pytest.raises(_lib.RldxError, match="static scratch"):
        _static(descs)
    torch.cuda.synchronize()
    assert int(out.count_nonzero()) == 0  # nothing was launched
