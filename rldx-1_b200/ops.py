"""Torch-facing wrappers of the per-op C-ABI entry points (device tensors in, device tensors out).

Each wrapper validates dtype/device/contiguity on the host, passes raw pointers to
librldx_b200.so on the current CUDA stream and raises RldxError on any failure.  They are what
the unit tests and the op-level drop-ins call; the control-step path runs inside the native
runtime (chain.py) instead.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import GemmDesc, check, load


def _p(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t: torch.Tensor, name: str, dtype=torch.bfloat16):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path exists)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def _row_major(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D row-major view")
    return t.stride(0)


def gemm_desc(
    x: torch.Tensor,
    weight: torch.Tensor,
    out: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    bias_mode: int = _lib.BIAS_FUSED,
    act: int = _lib.ACT_NONE,
    add: Optional[torch.Tensor] = None,
    add_row_mod: int = 0,
    epilogue: int = _lib.EPI_STORE,
    rows_in: int = 0,
    rows_out: int = 0,
    row_skip: int = 0,
    dt: float = 0.0,
    cat_ids: Optional[torch.Tensor] = None,
    rows_per_cat: int = 0,
    col_off: int = 0,
    tile_n: int = 0,
) -> GemmDesc:
    """Describes out = epilogue(x @ weight^T).  weight is [N, K] or [cats, N, K] (with cat_ids)."""
    _need(x, "x")
    _need(weight, "weight")
    _need(out, "out")
    lda = _row_major(x, "x")
    M, K = x.shape
    d = GemmDesc()
    d.a, d.lda, d.M, d.K = x.data_ptr(), lda, M, K
    d.b = weight.data_ptr()
    if cat_ids is not None:
        if weight.dim() != 3 or not weight.is_contiguous():
            raise ValueError("category weight must be a contiguous [cats, N, K] tensor")
        _need(cat_ids, "cat_ids", torch.int64)
        d.cat_ids, d.rows_per_cat, d.num_cats = cat_ids.data_ptr(), rows_per_cat, weight.shape[0]
        d.N, d.ldb, d.b_cat_stride = weight.shape[1], weight.shape[2], weight.shape[1] * weight.shape[2]
        if bias is not None:
            d.bias_cat_stride = bias.shape[-1]
    else:
        d.ldb = _row_major(weight, "weight")
        d.N = weight.shape[0]
    if bias is not None:
        _need(bias, "bias")
        d.bias, d.bias_mode = bias.data_ptr(), bias_mode
    d.act = act
    if add is not None:
        _need(add, "add")
        d.add, d.ld_add, d.add_row_mod = add.data_ptr(), _row_major(add, "add"), add_row_mod
    d.out, d.ldo, d.col_off = out.data_ptr(), _row_major(out, "out"), col_off
    d.epilogue, d.rows_in, d.rows_out, d.row_skip, d.dt = epilogue, rows_in, rows_out, row_skip, dt
    d.eps = 1e-6
    d.tile_n = tile_n
    return d


def gemm(descs: Sequence[GemmDesc], workspace: torch.Tensor = None) -> None:
    """Runs 1..4 GEMM problems in one grouped launch on the current stream.  With `workspace`
    (a zero-filled device byte tensor, at least gemm_workspace_size(descs) long) long K loops
    may be split across SMs; calls sharing a workspace must stay on one stream."""
    arr = (GemmDesc * len(descs))(*descs)
    if workspace is None:
        check(load().rldx_gemm(arr, len(descs), _stream()))
        return
    _need(workspace, "workspace", torch.uint8)
    check(load().rldx_gemm_ws(arr, len(descs), workspace.data_ptr(), workspace.numel(), _stream()))


def gemm_workspace_size(descs: Sequence[GemmDesc]) -> int:
    """Workspace bytes with which gemm(descs, workspace) would split K (0: no split)."""
    arr = (GemmDesc * len(descs))(*descs)
    n = C.c_uint64(0)
    check(load().rldx_gemm_workspace_size(arr, len(descs), C.byref(n)))
    return int(n.value)


def gemm_plan(descs: Sequence[GemmDesc]) -> dict:
    """The launch plan gemm(descs, workspace) uses: CTA pairs or single CTAs, CTAs, ring stages,
    the first problem's tile width and K splits."""
    arr = (GemmDesc * len(descs))(*descs)
    v = (C.c_int * 5)()
    check(load().rldx_gemm_plan(arr, len(descs), v))
    return {"pair": bool(v[0]), "ctas": v[1], "stages": v[2], "tile_n": v[3], "splits": v[4]}


def linear(x, weight, bias=None, *, act=_lib.ACT_NONE, bias_mode=_lib.BIAS_FUSED, add=None,
           out=None, tile_n=0) -> torch.Tensor:
    """nn.Linear (+activation, +residual) through the tcgen05 GEMM."""
    if out is None:
        out = torch.empty(x.shape[0], weight.shape[0], dtype=torch.bfloat16, device=x.device)
    gemm([gemm_desc(x, weight, out, bias, bias_mode=bias_mode, act=act, add=add, tile_n=tile_n)])
    return out


def qkv_desc(x, weight, bias, q_norm, k_norm, rope_cos, rope_sin, q, k, vt, *, tok_off: int,
             rows_per_batch: int, tile_n: int = 0, rope_identity: bool = False) -> GemmDesc:
    """QKV projection of one stream with fused per-head RMSNorm + RoPE, scattered into the joint
    attention layout q, k [B, H, L, 64] and vt [B, H, 64, Lp]."""
    B, H, L, hd = q.shape
    if hd != 64:
        raise ValueError("head_dim must be 64")
    d = gemm_desc(x, weight, q.view(-1, 64), bias, epilogue=_lib.EPI_QKV, rows_in=rows_per_batch,
                  rows_out=rows_per_batch, tile_n=tile_n)
    _need(q_norm, "q_norm")
    _need(k_norm, "k_norm")
    _need(rope_cos, "rope_cos", torch.float32)
    _need(rope_sin, "rope_sin", torch.float32)
    d.q_norm_w, d.k_norm_w = q_norm.data_ptr(), k_norm.data_ptr()
    d.rope_cos, d.rope_sin = rope_cos.data_ptr(), rope_sin.data_ptr()
    d.q, d.k, d.vt = q.data_ptr(), k.data_ptr(), vt.data_ptr()
    d.L, d.Lp, d.H, d.tok_off = L, vt.shape[-1], H, tok_off
    d.rope_identity = 1 if rope_identity else 0
    return d


def joint_attention(q, k, vt, seg_lens: Sequence[int], key_mask=None, outs=None, tiles_per_cta: int = 0):
    """Non-causal joint attention over concatenated segments (q, k [B, H, L, d], vt [B, H, d, Lp],
    d = 64 or 128); returns one output per segment as [B * seg_len, H * d]."""
    for t, n in ((q, "q"), (k, "k"), (vt, "vt")):
        _need(t, n)
        if not t.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
    B, H, L, hd = q.shape
    Lp = vt.shape[-1]
    if outs is None:
        outs = [torch.empty(B * n, H * hd, dtype=torch.bfloat16, device=q.device) for n in seg_lens]
    ptrs = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    lens = (C.c_int * len(seg_lens))(*seg_lens)
    if key_mask is not None:
        _need(key_mask, "key_mask", torch.uint8)
    check(load().rldx_joint_attention(_p(q), _p(k), _p(vt), B, H, L, Lp, hd, _p(key_mask), ptrs, lens,
                                      len(seg_lens), tiles_per_cta, _stream()))
    return outs


def attention(q, k, vt, seg_lens: Sequence[int] = None, *, causal: bool = False, key_mask=None,
              outs=None, tiles_per_cta: int = 0):
    """Attention through rldx_attention: q [B, H, L, d], k [B, Hkv, L, d], vt [B, Hkv, d, Lp]
    (Hkv divides H: grouped-query heads), optional causal mask; returns one output per segment
    as [B * seg_len, H * d] (one segment of L rows by default)."""
    for t, n in ((q, "q"), (k, "k"), (vt, "vt")):
        _need(t, n)
        if not t.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
    B, H, L, hd = q.shape
    seg_lens = list(seg_lens) if seg_lens is not None else [L]
    if outs is None:
        outs = [torch.empty(B * n, H * hd, dtype=torch.bfloat16, device=q.device) for n in seg_lens]
    d = _lib.AttentionDesc()
    d.q, d.k, d.vt = q.data_ptr(), k.data_ptr(), vt.data_ptr()
    d.B, d.H, d.kv_heads, d.L, d.Lp, d.head_dim = B, H, k.shape[1], L, vt.shape[-1], hd
    d.causal, d.tiles_per_cta = 1 if causal else 0, tiles_per_cta
    if key_mask is not None:
        _need(key_mask, "key_mask", torch.uint8)
        d.key_mask = key_mask.data_ptr()
    for i, (o, n) in enumerate(zip(outs, seg_lens)):
        d.out[i], d.seg_len[i], d.out_ld[i] = o.data_ptr(), n, _row_major(o, "out")
    d.nseg = len(seg_lens)
    check(load().rldx_attention(C.byref(d), _stream()))
    return outs


def layernorm(x, eps: float = 1e-6, scale1p=None, shift=None, out=None):
    """LayerNorm without affine (optionally * scale1p + shift) over the last dim of [rows, D]."""
    _need(x, "x")
    ld = _row_major(x, "x")
    if out is None:
        out = torch.empty_like(x)
    check(load().rldx_layernorm(_p(x), ld, _p(out), _row_major(out, "out"), x.shape[0], x.shape[1],
                                eps, _p(scale1p), _p(shift), _stream()))
    return out


def qk_rmsnorm_rope(x, weight, pos, cos_table, sin_table, eps: float = 1e-6, out=None):
    """Qwen3-style per-head RMSNorm + rotate-half RoPE on [T, H, 128]."""
    _need(x, "x")
    _need(pos, "pos", torch.int32)
    if not x.is_contiguous() or x.dim() != 3:
        raise ValueError("x must be contiguous [T, H, head_dim]")
    if out is None:
        out = torch.empty_like(x)
    T, Hh, hd = x.shape
    check(load().rldx_qk_rmsnorm_rope(_p(x), _p(out), _p(weight), _p(pos), _p(cos_table),
                                      _p(sin_table), T, Hh, hd, eps, _stream()))
    return out


def swiglu(gate, up, out=None):
    """silu(gate) * up for [rows, H] views (gate / up may be halves of one [rows, 2H] tensor)."""
    _need(gate, "gate")
    _need(up, "up")
    ld_g, ld_u = _row_major(gate, "gate"), _row_major(up, "up")
    if ld_g != ld_u:
        raise ValueError("gate and up must share a row stride")
    rows, H = gate.shape
    if out is None:
        out = torch.empty(rows, H, dtype=torch.bfloat16, device=gate.device)
    check(load().rldx_swiglu(_p(gate), _p(up), ld_g, _p(out), _row_major(out, "out"), rows, H,
                             _stream()))
    return out


def qkv_prep(segments, q, k, vt, eps: float = 1e-6) -> None:
    """Per-head QK RMSNorm + interleaved-pair RoPE of projected [q | k | v] rows into the joint
    attention layout q, k [B, H, L, 64] and vt [B, H, 64, Lp].  `segments` lists, in joint order,
    dicts with qkv ([rows, 3*H*64] or [B, rows, 3*H*64]), q_norm, k_norm and optionally
    rope_cos / rope_sin ([rows - rope_from, 32] fp32) and rope_from."""
    for t, n in ((q, "q"), (k, "k"), (vt, "vt")):
        _need(t, n)
    B, H, L, _ = q.shape
    Lp = vt.shape[-1]
    arr = (_lib.QkvSegment * len(segments))()
    keep = []
    for i, sg in enumerate(segments):
        x = sg["qkv"]
        _need(x, "qkv")
        if x.stride(-1) != 1:
            raise ValueError("qkv rows must be row-major")
        rows = x.shape[-2]
        arr[i].qkv, arr[i].ld, arr[i].rows = x.data_ptr(), x.stride(-2), rows
        arr[i].batch_stride = x.stride(0) if x.dim() == 3 else rows * x.stride(-2)
        qn, kn = sg["q_norm"].contiguous(), sg["k_norm"].contiguous()
        keep += [qn, kn]
        arr[i].q_norm, arr[i].k_norm = qn.data_ptr(), kn.data_ptr()
        if sg.get("rope_cos") is not None:
            c = sg["rope_cos"].float().contiguous()
            sn = sg["rope_sin"].float().contiguous()
            keep += [c, sn]
            arr[i].rope_cos, arr[i].rope_sin = c.data_ptr(), sn.data_ptr()
            arr[i].rope_from = int(sg.get("rope_from", 0))
    check(load().rldx_qkv_prep(arr, len(segments), B, H, L, Lp, eps, _p(q), _p(k), _p(vt), _stream()))


def res_layernorm(segments, *, fp32_sum: bool = False, eps: float = 1e-6) -> None:
    """sum = x (+ y) (+ v1) (+ v2) then LayerNorm, for up to 2 row groups in one launch.
    `segments`: dicts with x, ln_out and optionally y, v1, v2, sum_out ([rows, D] row-major views,
    vectors [D]).  fp32_sum False: bf16 rounding after each add in the order x, v1, v2, y;
    True: one fp32 sum."""
    arr = (_lib.ResLnSegment * len(segments))()
    for i, sg in enumerate(segments):
        x = sg["x"]
        _need(x, "x")
        ld = _row_major(x, "x")
        arr[i].x, arr[i].rows, arr[i].D, arr[i].ld = x.data_ptr(), x.shape[0], x.shape[1], ld
        for name in ("y", "v1", "v2", "sum_out", "ln_out"):
            t = sg.get(name)
            if t is None:
                continue
            _need(t, name)
            if name in ("y", "sum_out", "ln_out") and _row_major(t, name) != ld:
                raise ValueError(f"{name} must share the row stride of x")
            setattr(arr[i], name, t.data_ptr())
    check(load().rldx_res_layernorm(arr, len(segments), 1 if fp32_sum else 0, eps, _stream()))


def swiglu_bias(segments) -> None:
    """out = silu(gate + bias_gate) * (up + bias_up) in fp32, for up to 2 row groups.
    `segments`: dicts with gate, up ([rows, H] views sharing a row stride), bias_gate, bias_up
    ([H]) and out ([rows, H])."""
    arr = (_lib.SwigluBiasSegment * len(segments))()
    for i, sg in enumerate(segments):
        g, u, o = sg["gate"], sg["up"], sg["out"]
        for t, n in ((g, "gate"), (u, "up"), (o, "out"), (sg["bias_gate"], "bias_gate"), (sg["bias_up"], "bias_up")):
            _need(t, n)
        ld = _row_major(g, "gate")
        if _row_major(u, "up") != ld:
            raise ValueError("gate and up must share a row stride")
        arr[i].gate, arr[i].up, arr[i].out = g.data_ptr(), u.data_ptr(), o.data_ptr()
        arr[i].bias_gate, arr[i].bias_up = sg["bias_gate"].data_ptr(), sg["bias_up"].data_ptr()
        arr[i].ld_in, arr[i].ld_out = ld, _row_major(o, "out")
        arr[i].rows, arr[i].H = g.shape[0], g.shape[1]
    check(load().rldx_swiglu_bias(arr, len(segments), _stream()))


def device_error() -> int:
    """Reads and clears the device-side error word (synchronizes)."""
    v = C.c_uint(0)
    check(load().rldx_get_device_error(C.byref(v)))
    return int(v.value)


def set_wait_limit(cycles: int) -> None:
    """Bound of every in-kernel wait in SM cycles (current device)."""
    check(load().rldx_set_wait_limit(int(cycles)))


def get_wait_limit() -> int:
    v = C.c_int64(0)
    check(load().rldx_get_wait_limit(C.byref(v)))
    return int(v.value)


def wait_selftest(limit_cycles: int) -> None:
    """Launches the bounded-wait self-test on the current stream: a wait on a barrier nothing
    arrives on runs out after `limit_cycles` and records device error 0x400."""
    check(load().rldx_wait_selftest(int(limit_cycles), _stream()))
