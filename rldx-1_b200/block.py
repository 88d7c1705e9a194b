"""One joint MSAT block on the native kernels: the block-level counterpart of the reference's
ExpandedDoubleStreamBlock (rldx/model/modules/action_model/blocks.py:705-891, identity
modulation under temb_type="input_token", blocks.py:737-760).

    blk = B200ExpandedDoubleStreamBlock(block, device="cuda:0")
    sa, vl, p = blk(sa, vl, p, pe)          # bf16 [B, n, D] streams, pe = RoPE table [1|B, L, hd/2]

`pe` is the reference's RoPEEmbedder1D output over the joint [VL | SA | P] token order: complex
(full interleaved-pair rotation) or real (the bf16-cast module's cos-only table, the reference
quirk of rldx/inference/utils/loader.py:170).  Per stream: LayerNorm (no affine, eps 1e-6) ->
QKV GEMM with the per-head RMSNorm + RoPE epilogue scattering into the joint attention layout ->
joint attention over [VL | SA | P] -> output projection with the residual added in the GEMM
epilogue -> LayerNorm -> w12 GEMM with the SwiGLU epilogue (rows regrouped as [32 gate | 32 up])
-> w3 GEMM with the residual.  The three streams of each projection run as one grouped launch.
This is BASELINE config 1's block (cognition 256, action 16, physics 16, hidden 1024, 16 x 64
heads, SwiGLU 2816) on the GPU; the full control step runs the same kernels from the native
runtime (chain.py).
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib, ops

BF = torch.bfloat16


def swiglu_rows(hidden: int) -> torch.Tensor:
    """Row order of a w12 weight [2*hidden, D] that puts 32 gate rows next to the matching 32 up
    rows (the SwiGLU epilogue's layout); hidden must be a multiple of 32."""
    if hidden % 32:
        raise ValueError("SwiGLU hidden width must be a multiple of 32")
    return torch.cat([torch.cat([torch.arange(g * 32, g * 32 + 32), hidden + torch.arange(g * 32, g * 32 + 32)])
                      for g in range(hidden // 32)])


class B200ExpandedDoubleStreamBlock(nn.Module):
    STREAMS = ("vl", "sa", "p")  # joint token order

    def __init__(self, block: nn.Module, device=None, *, use_graph: bool = False):
        super().__init__()
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.heads = int(block.num_heads)
        self.w = {}
        for s in self.STREAMS:
            qkv, proj, mlp = getattr(block, f"{s}_qkv"), getattr(block, f"{s}_proj"), getattr(block, f"{s}_mlp")
            hid = mlp.w12.weight.shape[0] // 2
            idx = swiglu_rows(hid)
            cvt = lambda t: t.detach().to(self.device, BF).contiguous()  # noqa: E731
            self.w[s] = {
                "qkv": cvt(qkv.weight), "qkv_b": cvt(qkv.bias),
                "qn": cvt(getattr(block, f"q_norm_{s}").weight), "kn": cvt(getattr(block, f"k_norm_{s}").weight),
                "proj": cvt(proj.weight), "proj_b": cvt(proj.bias),
                "w12": cvt(mlp.w12.weight[idx]), "w12_b": cvt(mlp.w12.bias[idx]),
                "w3": cvt(mlp.w3.weight), "w3_b": cvt(mlp.w3.bias), "hidden": hid,
            }
        self.head_dim = self.w["sa"]["qn"].shape[0]
        if self.head_dim != 64:
            raise NotImplementedError("the block's QKV epilogue handles 64-dim heads")
        self.use_graph = use_graph
        self._bound = None
        self._graph = None
        self._shapes = None

    def _bind(self, sa, vl, p):
        B = sa.shape[0]
        n = {"vl": vl.shape[1], "sa": sa.shape[1], "p": p.shape[1]}
        L = sum(n.values())
        Lp = (L + 7) // 8 * 8
        H, d = self.heads, self.head_dim
        dev = self.device
        st = {"n": n, "B": B, "L": L}
        st["x"] = {s: torch.empty(B * n[s], self.w[s]["proj"].shape[0], dtype=BF, device=dev) for s in self.STREAMS}
        st["y"] = {s: torch.empty_like(st["x"][s]) for s in self.STREAMS}
        st["h"] = {s: torch.empty(B * n[s], self.w[s]["hidden"], dtype=BF, device=dev) for s in self.STREAMS}
        st["o"] = {s: torch.empty(B * n[s], H * d, dtype=BF, device=dev) for s in self.STREAMS}
        st["q"] = torch.zeros(B, H, L, d, dtype=BF, device=dev)
        st["k"] = torch.zeros_like(st["q"])
        st["vt"] = torch.zeros(B, H, d, Lp, dtype=BF, device=dev)
        st["cos"] = torch.empty(L, d // 2, dtype=torch.float32, device=dev)
        st["sin"] = torch.empty_like(st["cos"])
        off, descs = 0, {"qkv": [], "proj": [], "w12": [], "w3": []}
        for s in self.STREAMS:
            w, x, y, h, o = self.w[s], st["x"][s], st["y"][s], st["h"][s], st["o"][s]
            descs["qkv"].append(ops.qkv_desc(y, w["qkv"], w["qkv_b"], w["qn"], w["kn"], st["cos"], st["sin"],
                                             st["q"], st["k"], st["vt"], tok_off=off, rows_per_batch=n[s]))
            descs["proj"].append(ops.gemm_desc(o, w["proj"], x, w["proj_b"], add=x))
            descs["w12"].append(ops.gemm_desc(y, w["w12"], h, w["w12_b"], epilogue=_lib.EPI_SWIGLU))
            descs["w3"].append(ops.gemm_desc(h, w["w3"], x, w["w3_b"], add=x))
            off += n[s]
        st["descs"] = descs
        st["ws"] = {}
        for key, ds in descs.items():
            need = ops.gemm_workspace_size(ds)
            st["ws"][key] = torch.zeros(need, dtype=torch.uint8, device=dev) if need else None
        self._bound = st

    def _run(self):
        st = self._bound
        for s in self.STREAMS:
            ops.layernorm(st["x"][s], out=st["y"][s])
        ops.gemm(st["descs"]["qkv"], st["ws"]["qkv"])
        ops.joint_attention(st["q"], st["k"], st["vt"], [st["n"][s] for s in self.STREAMS],
                            outs=[st["o"][s] for s in self.STREAMS])
        ops.gemm(st["descs"]["proj"], st["ws"]["proj"])
        for s in self.STREAMS:
            ops.layernorm(st["x"][s], out=st["y"][s])
        ops.gemm(st["descs"]["w12"], st["ws"]["w12"])
        ops.gemm(st["descs"]["w3"], st["ws"]["w3"])

    @property
    def launches(self) -> int:
        return 2 * len(self.STREAMS) + 5

    def _load(self, sa, vl, p):
        st = self._bound
        for s, t in (("vl", vl), ("sa", sa), ("p", p)):
            st["x"][s].copy_(t.reshape(-1, t.shape[-1]))

    def forward(self, sa: torch.Tensor, vl: torch.Tensor, p: torch.Tensor, pe: torch.Tensor):
        shapes = (tuple(sa.shape), tuple(vl.shape), tuple(p.shape))
        if self._bound is None:
            self._bind(sa, vl, p)
            self._shapes = shapes
        elif shapes != self._shapes:
            raise ValueError(f"stream shapes {shapes} differ from the bound {self._shapes}")
        st = self._bound
        tab = pe[0] if pe.dim() == 3 else pe
        if tab.shape[0] != st["L"] or tab.shape[-1] != self.head_dim // 2:
            raise ValueError(f"pe must hold [L={st['L']}, {self.head_dim // 2}] entries")
        if torch.is_complex(tab):
            st["cos"].copy_(tab.real.float())
            st["sin"].copy_(tab.imag.float())
        else:  # bf16-cast module: cos-only rotation
            st["cos"].copy_(tab.float())
            st["sin"].zero_()
        self._load(sa, vl, p)
        if self.use_graph:
            if self._graph is None:
                side = torch.cuda.Stream(self.device)
                side.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(side):
                    self._run()  # warm-up outside capture (plans, tensor maps, kernel attributes)
                torch.cuda.current_stream(self.device).wait_stream(side)
                self._graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self._graph):
                    self._run()
                self._load(sa, vl, p)
            self._graph.replay()
        else:
            self._run()
        B = st["B"]
        return tuple(st["x"][s].view(B, st["n"][s], -1).clone() for s in ("sa", "vl", "p"))

    def replay(self) -> None:
        """Re-runs the bound block on its current buffers (timing)."""
        if self._graph is not None:
            self._graph.replay()
        else:
            self._run()
