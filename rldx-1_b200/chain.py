"""Drop-in replacements for the reference's action-head chains.

`B200ExpandedActionHeadChain` has the constructor and forward signature of
CustomExpandedActionHeadChain (rldx/inference/action_model/engine/custom_expanded_action_model_chain.py:19-213),
the all-modality head (ExpandedDoubleStreamBlocks over [VL | SA | P], then ExpandedSingleStreamBlocks
over [VL_proj | SA | P] when the model has any):

    chain = B200ExpandedActionHeadChain(gs_action_model, device, dtype=torch.bfloat16)
    actions = chain(vl_embs, state, embodiment_id, init_noise=None, physics_hist=None,
                    physics_init_noise=None)

`B200ActionHeadChain` has those of CustomActionHeadChain
(rldx/inference/action_model/engine/custom_action_model_chain.py:23-170), the head without add-ons
(DoubleStreamBlocks over [VL | SA] with a VL stream of its own width, vl_proj_to_sa, then
SingleStreamBlocks over [VL_proj | SA]):

    chain = B200ActionHeadChain(gs_action_model, device, dtype=torch.bfloat16)
    actions = chain(vl_embs, state, embodiment_id, init_noise=None)

Both take `prefix_actions` (B, prefix_len, action_dim) when the model was built for RTC trained
mode (`gs_action_model.prefix_len > 0`, or the `prefix_len=` argument): those actions stay locked
and are encoded at t = 1, as in GraphSafeActionModel.forward (graph_safe_action_model.py:196-300).

It reads the weights by the reference's attribute names from a GraphSafeActionModel
(rldx/inference/action_model/model/graph_safe_action_model.py:27-168) or from an action model
exposing `.model` (MSAT), `.state_encoder`, `.action_encoder`, `.action_decoder`,
`.position_embedding` and `.physics` (RLDXActionModel, rldx/model/core/rldx.py:30-106), and
hands them to the native runtime (rldx_msat_create), which copies them into its own device
arena, bakes the step-constant tables and captures the control step as one CUDA graph.  The
native handle is created on the first forward, when the token counts are known (as the
reference's _CompiledDispatcher builds on its first call, rldx/inference/serve_optimization.py:432-511);
a later call with other shapes raises instead of falling back.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch
from torch import nn

from . import _lib
from ._lib import (BlockWeights, CatLinear, Linear, MsatConfig, MsatIO, MsatWeights,
                   SingleBlockWeights, StreamWeights, check)


def _parts(head: nn.Module):
    """(msat, state_encoder, action_encoder, action_decoder, position_embedding, physics, vlln);
    physics is None for a head without the physics stream."""
    if hasattr(head, "gs_msat"):  # GraphSafeActionModel
        msat = head.gs_msat._msat if hasattr(head.gs_msat, "_msat") else head.gs_msat
        physics = None
        if getattr(head, "physics_cond_encoder", None) is not None:
            physics = nn.Module()
            physics.physics_cond_encoder = head.physics_cond_encoder
            physics.physics_fut_encoder = head.physics_fut_encoder
            physics.physics_decoder = head.physics_decoder
            physics.physics_hist_len = head.physics_hist_len
            physics.physics_fut_len = head.physics_fut_len
            physics.physics_dim = head.physics_dim
    else:
        msat = head.model
        physics = getattr(head, "physics", None)
    if not getattr(msat, "use_physics", physics is not None):
        physics = None
    return (msat, head.state_encoder, head.action_encoder, head.action_decoder,
            head.position_embedding, physics, getattr(head, "vlln", nn.Identity()))


def _check_single_block(blk: nn.Module, prefix: str) -> None:
    """The runtime implements the SingleStreamBlock form the heads are built with: LayerNorm
    without affine as pre_norm, no post_norm, SwiGLU with mlp_proj (blocks.py:42-254)."""
    pre = getattr(blk, f"{prefix}pre_norm")
    if not isinstance(pre, nn.LayerNorm) or pre.weight is not None:
        raise NotImplementedError("single blocks: only a LayerNorm without affine as pre_norm is bound")
    if not isinstance(getattr(blk, f"{prefix}post_norm", nn.Identity()), nn.Identity):
        raise NotImplementedError("single blocks: post_norm must be the identity")
    if getattr(blk, f"{prefix}mlp_proj", None) is None:
        raise NotImplementedError("single blocks: the SwiGLU form with mlp_proj is the one bound")
    if getattr(blk, f"{prefix}linear1").bias is None or getattr(blk, f"{prefix}linear2").bias is None:
        raise NotImplementedError("single blocks: linear1 / linear2 without bias are not bound")


class _B200HeadChain(nn.Module):
    """State encoder (+ physics history encoder), then num_steps x [action (+ physics) encoders
    + MSAT + decoders + Euler], as one native control step on librldx_b200."""

    _physics = True

    def __init__(self, gs_action_model: nn.Module, device=None, dtype=torch.bfloat16, *,
                 num_inference_timesteps: Optional[int] = None, use_graph: bool = True,
                 prefix_len: Optional[int] = None):
        super().__init__()
        if dtype != torch.bfloat16:
            raise ValueError("the B200 chain computes in bfloat16 only")
        parts = _parts(gs_action_model)
        self._msat, self._state_enc, self._act_enc, self._act_dec, self._pos, self._phys, vlln = parts
        if (self._phys is not None) != self._physics:
            raise ValueError(f"{type(self).__name__} needs a head {'with' if self._physics else 'without'} "
                             "the physics stream")
        if not isinstance(vlln, nn.Identity):
            raise NotImplementedError("use_vlln=True (LayerNorm on backbone features) is not bound")
        for blk in getattr(self._msat, "single_blocks", []):
            _check_single_block(blk, "")
            if self._physics:
                _check_single_block(blk, "p_")
        if getattr(self._msat, "temb_type", "input_token") != "input_token":
            raise NotImplementedError("only temb_type='input_token' is supported")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.num_inference_timesteps = int(num_inference_timesteps or getattr(
            gs_action_model, "num_inference_timesteps", 4))
        self.action_horizon = getattr(gs_action_model, "action_horizon", None)
        self.action_dim = self._act_dec.layer2.W.shape[2]
        # RTC trained-mode prefix length, baked into the native plan (the reference bakes it into
        # its chain: custom_action_model_chain.py:31-35)
        self.prefix_len = int(prefix_len if prefix_len is not None else getattr(gs_action_model, "prefix_len", 0))
        self.use_graph = use_graph
        self._handle = None
        self._shapes = None
        self._keep = []

    # ------------------------------------------------------------------ binding
    def _bf16(self, t: torch.Tensor) -> int:
        t = t.detach().to(device=self.device, dtype=torch.bfloat16).contiguous()
        self._keep.append(t)
        return t.data_ptr()

    def _lin(self, m: nn.Module) -> Linear:
        return Linear(self._bf16(m.weight), self._bf16(m.bias))

    def _cat(self, m: nn.Module) -> CatLinear:
        return CatLinear(self._bf16(m.W), self._bf16(m.b))

    def _config(self, B, n_vl, n_state, horizon, hist, fut) -> MsatConfig:
        msat = self._msat
        blk = msat.double_blocks[0]
        rope = msat.rope_embedder
        mode = getattr(msat, "positional_embeddings", "rope_sa_only")
        if mode not in ("rope_sa_only", "rope_vl_sa"):
            raise NotImplementedError(f"positional_embeddings={mode!r} is not supported")
        c = MsatConfig()
        c.batch, c.n_vl, c.n_state, c.horizon = B, n_vl, n_state, horizon
        c.physics_hist, c.physics_fut = hist, fut
        c.dim = blk.sa_qkv.weight.shape[1]
        c.heads = blk.num_heads
        c.head_dim = blk.q_norm_sa.weight.shape[0]
        c.depth = len(msat.double_blocks)
        c.mlp_hidden = blk.sa_mlp.w3.weight.shape[1]
        c.vl_mlp_hidden = blk.vl_mlp.w3.weight.shape[1]
        c.out_dim = msat.proj_out_2.weight.shape[0]
        c.action_dim = self._act_dec.layer2.W.shape[2]
        c.state_dim = self._state_enc.layer1.W.shape[1]
        c.dec_hidden = self._state_enc.layer1.W.shape[2]
        c.physics_dim = self._phys.physics_cond_encoder.W1.weight.shape[1] if self._physics else 0
        c.standard_path = 0 if self._physics else 1
        c.vl_dim = blk.vl_qkv.weight.shape[1]
        singles = list(getattr(msat, "single_blocks", []))
        c.depth_single = len(singles)
        if singles:
            c.single_expanded = singles[0].mlp_proj.weight.shape[1]
            c.single_mlp_hidden = singles[0].mlp_proj.weight.shape[0]
        c.num_embodiments = self._state_enc.layer1.W.shape[0]
        c.num_steps = self.num_inference_timesteps
        c.rope_mode = _lib.ROPE_SA_ONLY if mode == "rope_sa_only" else _lib.ROPE_VL_SA
        # bf16-cast modules lost the imaginary part of the RoPE tables: cos-only rotation
        # (same detection as rldx/inference/action_model/engine/custom_msat_chain.py:50-54)
        c.rope_cos_only = 0 if rope.freqs_cis_0.is_complex() else 1
        c.rope_theta = float(rope.theta)
        c.rope_max_seq = int(rope.freqs_cis_0.shape[0])
        c.temb_channels = msat.timestep_encoder.timestep_embedder.linear_1.weight.shape[1]
        c.use_graph = 1 if self.use_graph else 0
        c.prefix_len = self.prefix_len
        c.key_mask = 1  # masked steps replay a second graph; unmasked ones pay nothing for it
        if not isinstance(getattr(msat, "time_token_proj", nn.Identity()), nn.Identity):
            raise NotImplementedError("time_token_proj must be the identity (inner_dim == sa_dim)")
        return c

    def _weights(self) -> MsatWeights:
        msat = self._msat
        w = MsatWeights()
        blocks = (BlockWeights * len(msat.double_blocks))()
        for i, blk in enumerate(msat.double_blocks):
            for s in (("vl", "sa", "p") if self._physics else ("vl", "sa")):
                sw = StreamWeights()
                sw.qkv = self._lin(getattr(blk, f"{s}_qkv"))
                sw.proj = self._lin(getattr(blk, f"{s}_proj"))
                mlp = getattr(blk, f"{s}_mlp")
                sw.w12 = self._lin(mlp.w12)
                sw.w3 = self._lin(mlp.w3)
                sw.q_norm = self._bf16(getattr(blk, f"q_norm_{s}").weight)
                sw.k_norm = self._bf16(getattr(blk, f"k_norm_{s}").weight)
                setattr(blocks[i], s, sw)
        self._keep.append(blocks)
        w.blocks = C.cast(blocks, C.POINTER(BlockWeights))
        singles = list(getattr(msat, "single_blocks", []))
        if singles:
            sb = (SingleBlockWeights * len(singles))()
            for i, blk in enumerate(singles):
                for pre in (("", "p_") if self._physics else ("",)):
                    setattr(sb[i], f"{pre}linear1", self._lin(getattr(blk, f"{pre}linear1")))
                    setattr(sb[i], f"{pre}linear2", self._lin(getattr(blk, f"{pre}linear2")))
                    setattr(sb[i], f"{pre}mlp_proj", self._lin(getattr(blk, f"{pre}mlp_proj")))
                    setattr(sb[i], f"{pre}q_norm", self._bf16(getattr(blk, f"{pre}q_norm").weight))
                    setattr(sb[i], f"{pre}k_norm", self._bf16(getattr(blk, f"{pre}k_norm").weight))
            self._keep.append(sb)
            w.single_blocks = C.cast(sb, C.POINTER(SingleBlockWeights))
            if not isinstance(msat.vl_proj_to_sa, nn.Identity):
                w.vl_proj_to_sa = self._lin(msat.vl_proj_to_sa)
        te = msat.timestep_encoder.timestep_embedder
        w.temb_lin1, w.temb_lin2 = self._lin(te.linear_1), self._lin(te.linear_2)
        w.proj_out_1, w.proj_out_2 = self._lin(msat.proj_out_1), self._lin(msat.proj_out_2)
        if self._physics:
            w.proj_out_phys_1 = self._lin(msat.proj_out_physics_1)
            w.proj_out_phys_2 = self._lin(msat.proj_out_physics_2)
        w.state_l1, w.state_l2 = self._cat(self._state_enc.layer1), self._cat(self._state_enc.layer2)
        ae = self._act_enc
        w.act_w1, w.act_w2, w.act_w3 = self._cat(ae.W1), self._cat(ae.W2), self._cat(ae.W3)
        w.dec_l1, w.dec_l2 = self._cat(self._act_dec.layer1), self._cat(self._act_dec.layer2)
        w.pos_emb = self._bf16(self._pos.weight)
        # the module's own RoPE tables (complex: full rotation; real: the cos the bf16 cast kept);
        # a module without both per-axis tables of the expected shape gets them computed
        rope = msat.rope_embedder
        mode = getattr(msat, "positional_embeddings", "rope_sa_only")
        axes = (16, 48) if mode == "rope_sa_only" else (48, 16)
        tabs = [getattr(rope, f"freqs_cis_{i}", None) for i in range(2)]
        n = int(tabs[0].shape[0]) if tabs[0] is not None else 0
        if all(t is not None and tuple(t.shape) == (n, a // 2) for t, a in zip(tabs, axes)):
            for i, t in enumerate(tabs):
                t = t.detach()
                cos = (t.real if t.is_complex() else t).to(self.device, torch.float32).contiguous()
                self._keep.append(cos)
                w.rope_cos[i] = cos.data_ptr()
                if t.is_complex():
                    sin = t.imag.to(self.device, torch.float32).contiguous()
                    self._keep.append(sin)
                    w.rope_sin[i] = sin.data_ptr()
        if not self._physics:
            return w
        pc, pf, pd = (self._phys.physics_cond_encoder, self._phys.physics_fut_encoder,
                      self._phys.physics_decoder)
        w.phc_w1, w.phc_w2, w.phc_w3 = self._lin(pc.W1), self._lin(pc.W2), self._lin(pc.W3)
        w.phf_w1, w.phf_w2, w.phf_w3 = self._lin(pf.W1), self._lin(pf.W2), self._lin(pf.W3)
        w.phd_l1, w.phd_l2 = self._lin(pd.net[0]), self._lin(pd.net[2])
        return w

    def bind(self, batch: int, n_vl: int, n_state: int, horizon: int, physics_hist: int,
             physics_fut: int) -> None:
        """Creates the native handle for these token counts (done by the first forward)."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            cfg = self._config(batch, n_vl, n_state, horizon, physics_hist, physics_fut)
            weights = self._weights()
            handle = C.c_void_p()
            rc = lib.rldx_msat_create(C.byref(cfg), C.byref(weights), C.byref(handle))
            self._keep.clear()  # the runtime copied every weight into its own arena
            check(rc)
        self._handle = handle
        self._shapes = (batch, n_vl, n_state, horizon, physics_hist, physics_fut)
        self._cfg = cfg

    @property
    def launches_per_step(self) -> int:
        return int(_lib.load().rldx_msat_launch_count(self._handle)) if self._handle else 0

    # ------------------------------------------------------------------ forward
    def _step(self, vl_embs, state, embodiment_id, init_noise, physics_hist, physics_init_noise,
              prefix_actions, vl_attention_mask=None, physics_attention_mask=None):
        B, n_vl, _ = vl_embs.shape
        if self.prefix_len and prefix_actions is None:
            raise ValueError(f"this chain was built with prefix_len={self.prefix_len}: prefix_actions is required")
        if state.dim() == 2:
            state = state.unsqueeze(1)
        horizon = self.action_horizon or (init_noise.shape[1] if init_noise is not None else 16)
        hist = physics_hist.shape[1] if self._physics else 0
        fut = (physics_init_noise.shape[1] if physics_init_noise is not None else horizon) if self._physics else 0
        shapes = (B, n_vl, state.shape[1], horizon, hist, fut)
        if self._handle is None:
            self.bind(*shapes)
        elif shapes != self._shapes:
            raise ValueError(f"input shapes {shapes} differ from the bound shapes {self._shapes}")
        dev = self.device
        bf = torch.bfloat16

        def _in(t, dtype=bf):
            if t.device != dev or t.dtype != dtype or not t.is_contiguous():
                t = t.to(device=dev, dtype=dtype).contiguous()
            return t

        vl = _in(vl_embs)
        st = _in(state)
        ids = _in(embodiment_id.reshape(-1), torch.int64)
        if init_noise is None:
            init_noise = torch.randn(B, horizon, self.action_dim, dtype=bf, device=dev)
        noise = _in(init_noise)
        ph_ptr = pn_ptr = None
        if self._physics:
            if physics_init_noise is None:
                physics_init_noise = torch.randn(B, fut, self._cfg.physics_dim, dtype=bf, device=dev)
            ph, pn = _in(physics_hist), _in(physics_init_noise)
            ph_ptr, pn_ptr = ph.data_ptr(), pn.data_ptr()
        pre_ptr = None
        if self.prefix_len:
            if tuple(prefix_actions.shape) != (B, self.prefix_len, self.action_dim):
                raise ValueError(f"prefix_actions must be {(B, self.prefix_len, self.action_dim)}, "
                                 f"got {tuple(prefix_actions.shape)}")
            pre = _in(prefix_actions)
            pre_ptr = pre.data_ptr()
        vm_ptr = pm_ptr = None
        if vl_attention_mask is not None:
            vm = _in((vl_attention_mask != 0).reshape(B, n_vl), torch.uint8)
            vm_ptr = vm.data_ptr()
        if physics_attention_mask is not None:
            if not self._physics:
                raise ValueError("physics_attention_mask needs the physics stream")
            pm = _in((physics_attention_mask != 0).reshape(B), torch.uint8)
            pm_ptr = pm.data_ptr()
        out = torch.empty(B, horizon, self.action_dim, dtype=bf, device=dev)
        io = MsatIO(vl.data_ptr(), st.data_ptr(), ids.data_ptr(), noise.data_ptr(), ph_ptr,
                    pn_ptr, out.data_ptr(), pre_ptr, vm_ptr, pm_ptr)
        stream = torch.cuda.current_stream(dev)
        # a device error recorded by an earlier (asynchronous) step surfaces here, before more
        # work is queued behind it
        self._raise_on_device_error(wait=False)
        check(_lib.load().rldx_msat_step(self._handle, C.byref(io), C.c_void_p(stream.cuda_stream)))
        return out

    def _raise_on_device_error(self, wait: bool) -> None:
        code = self.device_status(wait)
        if code:
            raise _lib.RldxError(_lib.RLDX_ERR_DEVICE, f"device error 0x{code:x} recorded by a control step")

    def device_status(self, wait: bool = True) -> int:
        """Device error code of the last control step (0: none; with wait=False, 0 while it is
        still running).  Reading clears it."""
        if self._handle is None:
            return 0
        code = C.c_uint(0)
        check(_lib.load().rldx_msat_status(self._handle, 1 if wait else 0, C.byref(code)))
        return int(code.value)

    def block_end(self, step: int, block: int) -> int:
        """Launches from the start of a control step through the last one of `block` (double
        blocks, then single blocks) of Euler step `step`."""
        n = C.c_int(0)
        check(_lib.load().rldx_msat_block_end(self._handle, step, block, C.byref(n)))
        return int(n.value)

    def run_partial(self, inp: dict, n_ops: int) -> None:
        """Runs the first n_ops launches of a control step on device inputs (read_buffer then
        shows the residual streams at that point)."""
        out = torch.empty(inp["init_noise"].shape, dtype=torch.bfloat16, device=self.device)
        io = self._io(inp, out)
        stream = torch.cuda.current_stream(self.device)
        check(_lib.load().rldx_msat_run_partial(self._handle, C.byref(io), n_ops,
                                                C.c_void_p(stream.cuda_stream)))

    def _io(self, inp: dict, out: torch.Tensor) -> MsatIO:
        ph = inp["physics_hist"].data_ptr() if self._physics else None
        pn = inp["physics_noise"].data_ptr() if self._physics else None
        pre = inp["prefix_actions"].data_ptr() if self.prefix_len else None
        vm = inp["vl_mask"].data_ptr() if inp.get("vl_mask") is not None else None  # uint8 [B, n_vl]
        pm = inp["physics_mask"].data_ptr() if inp.get("physics_mask") is not None else None  # uint8 [B]
        return MsatIO(inp["vl"].data_ptr(), inp["state"].data_ptr(), inp["embodiment_id"].data_ptr(),
                      inp["init_noise"].data_ptr(), ph, pn, out.data_ptr(), pre, vm, pm)

    def forward_host(self, inp: dict, out: torch.Tensor) -> torch.Tensor:
        """One control step from (pinned) host tensors to a host tensor through
        rldx_msat_step_host: host->device copies, the captured graph, device->host copy and a
        stream synchronize.  `inp` holds the forward() arguments as contiguous CPU tensors."""
        if self._handle is None:
            raise RuntimeError("bind() or run forward() once before forward_host()")
        io = self._io(inp, out)
        stream = torch.cuda.current_stream(self.device)
        check(_lib.load().rldx_msat_step_host(self._handle, C.byref(io), C.c_void_p(stream.cuda_stream)))
        return out

    def profile(self, inp: dict) -> list:
        """Per-launch device times of one eager control step: [(kind, grid, ms, bytes, flops)]."""
        lib = _lib.load()
        n = self.launches_per_step
        arr = (_lib.OpProfile * n)()
        got = C.c_int(0)
        out = torch.empty(inp["init_noise"].shape, dtype=torch.bfloat16, device=self.device)
        io = self._io(inp, out)
        stream = torch.cuda.current_stream(self.device)
        check(lib.rldx_msat_profile(self._handle, C.byref(io), arr, n, C.byref(got),
                                    C.c_void_p(stream.cuda_stream)))
        kinds = ("gemm", "attention", "layernorm", "copy", "status")
        return [(kinds[a.kind], a.grid, a.ms, a.bytes, a.flops) for a in arr[:got.value]]

    def read_buffer(self, which: int) -> torch.Tensor:
        """Copy of a runtime buffer of the last step (0 X_vl, 1 X_sa, 2 X_p, 3 actions)."""
        lib = _lib.load()
        rows, cols = C.c_int64(), C.c_int64()
        check(lib.rldx_msat_read_buffer(self._handle, which, None, 0, C.byref(rows), C.byref(cols), None))
        out = torch.empty(rows.value, cols.value, dtype=torch.bfloat16, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        check(lib.rldx_msat_read_buffer(self._handle, which, C.c_void_p(out.data_ptr()),
                                        out.numel() * 2, C.byref(rows), C.byref(cols),
                                        C.c_void_p(stream.cuda_stream)))
        return out

    def __del__(self):
        # plain dict access: nn.Module.__setattr__ may be unusable during interpreter shutdown
        h = self.__dict__.pop("_handle", None)
        if h:
            try:
                _lib.load().rldx_msat_destroy(h)
            except Exception:  # noqa: BLE001
                pass


class B200ExpandedActionHeadChain(_B200HeadChain):
    """All-modality head: CustomExpandedActionHeadChain.forward
    (custom_expanded_action_model_chain.py:82-213)."""

    _physics = True

    def forward(self, vl_embs, state, embodiment_id, init_noise=None, physics_hist=None,
                physics_init_noise=None, prefix_actions=None, vl_attention_mask=None,
                physics_attention_mask=None):
        """vl_attention_mask [B, n_vl] (1 = visible) / physics_attention_mask [B]: key masks of the
        backbone tokens and of each observation's physics tokens, as the reference passes
        backbone_attention_mask and physics_mask to MSAT (rldx/model/core/rldx.py:619-621, 660-666);
        the reference's graph-safe chains take no masks."""
        if physics_hist is None:
            raise ValueError("physics_hist is required by the all-modality chain")
        return self._step(vl_embs, state, embodiment_id, init_noise, physics_hist, physics_init_noise,
                          prefix_actions, vl_attention_mask, physics_attention_mask)


class B200ActionHeadChain(_B200HeadChain):
    """Head without add-ons: CustomActionHeadChain.forward (custom_action_model_chain.py:81-170)."""

    _physics = False

    def forward(self, vl_embs, state, embodiment_id, init_noise=None, prefix_actions=None,
                vl_attention_mask=None, **kwargs):
        """vl_attention_mask [B, n_vl] (1 = visible): key mask of the backbone tokens
        (rldx/model/core/rldx.py:619-621)."""
        return self._step(vl_embs, state, embodiment_id, init_noise, None, None, prefix_actions,
                          vl_attention_mask)
