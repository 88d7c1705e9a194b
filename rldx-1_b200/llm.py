"""Drop-in replacement for the reference's VLM backbone LLM chain.

`B200LLMChain` has the constructor and forward of CustomLLMChain
(rldx/inference/backbone/llm/engine/custom_llm_chain.py:63-170):

    chain = B200LLMChain(decoder_layers, norm, pos_cos, signed_sin, apply_final_norm=True)
    hidden = chain(hidden_states)            # [B, M, hidden] bf16 -> [B, M, hidden] bf16

`decoder_layers` are Qwen3 text decoder layers (the reference's vendored
Qwen3VLTextDecoderLayer, rldx/model/modules/backbone/modeling_qwen3_vl.py:509-560, or anything
with the same attribute names; a video-token-compression LayerWrapper is unwrapped as the
reference unwraps it), `norm` the final RMSNorm, `pos_cos` / `signed_sin` the [M, head_dim] RoPE
tables of the reference chain (signed_sin carries rotate_half's sign:
-sin on the first half, fused_llm_attention.py:787-795).  The weights are copied into the
native runtime (rldx_llm_create) on the first forward, when the batch size is known; the stack
then runs as one CUDA graph of hand-written sm_100a kernels.  Deepstack feature injection is
not bound (the reference adds it for the first layers of its vision-language path).
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch
from torch import nn

from . import _lib
from ._lib import LlmConfig, LlmLayerWeights, LlmWeights, check


def _raw_layer(layer: nn.Module) -> nn.Module:
    """A video-token-compression LayerWrapper wraps the decoder layer (custom_llm_chain.py:36-40)."""
    if hasattr(layer, "layer") and hasattr(layer, "internal_projection"):
        return layer.layer
    return layer


def unsigned_sin(signed_sin: torch.Tensor) -> torch.Tensor:
    half = signed_sin.shape[-1] // 2
    sin = signed_sin.clone()
    sin[..., :half] = -sin[..., :half]
    return sin


class B200LLMChain(nn.Module):
    """norm_weight_first / causal_block select the memory module's variant (see
    B200MemoryChain); a layer without q_norm / k_norm runs without the per-head QK RMSNorm."""

    def __init__(self, layers, norm: nn.Module, pos_cos: torch.Tensor, signed_sin: torch.Tensor,
                 apply_final_norm: bool = True, *, device=None, use_graph: bool = True,
                 norm_weight_first: bool = False, causal_block: int = 1):
        super().__init__()
        self.layers = [_raw_layer(layer) for layer in layers]
        if not self.layers:
            raise ValueError("B200LLMChain needs at least one decoder layer")
        self.norm = norm
        self.apply_final_norm = apply_final_norm
        self.device = torch.device(device) if device is not None else pos_cos.device
        if self.device.type != "cuda":
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.cos = pos_cos.detach().to(self.device, torch.bfloat16).contiguous()
        self.sin = unsigned_sin(signed_sin.detach()).to(self.device, torch.bfloat16).contiguous()
        attn = self.layers[0].self_attn
        self.qk_norm = getattr(attn, "q_norm", None) is not None
        self.head_dim = attn.q_norm.weight.shape[0] if self.qk_norm else int(attn.head_dim)
        self.q_heads = attn.q_proj.weight.shape[0] // self.head_dim
        self.kv_heads = attn.k_proj.weight.shape[0] // self.head_dim
        self.hidden = attn.q_proj.weight.shape[1]
        self.ffn = self.layers[0].mlp.gate_proj.weight.shape[0]
        ln = self.layers[0].input_layernorm
        self.eps = float(getattr(ln, "variance_epsilon", getattr(ln, "eps", 1e-6)))
        self.norm_weight_first = norm_weight_first
        self.causal_block = int(causal_block)
        for layer in self.layers:
            a = layer.self_attn
            for lin in (a.q_proj, a.k_proj, a.v_proj, a.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj,
                        layer.mlp.down_proj):
                if getattr(lin, "bias", None) is not None:
                    raise NotImplementedError("Qwen3 projections have no bias; a biased layer is not bound")
        self.use_graph = use_graph
        self._handle = None
        self._batch = None
        self._keep = []

    def _bf16(self, t: torch.Tensor) -> int:
        t = t.detach().to(device=self.device, dtype=torch.bfloat16).contiguous()
        self._keep.append(t)
        return t.data_ptr()

    def bind(self, batch: int) -> None:
        M = self.cos.shape[0]
        cfg = LlmConfig(batch=batch, tokens=M, hidden=self.hidden, q_heads=self.q_heads, kv_heads=self.kv_heads,
                        head_dim=self.head_dim, ffn=self.ffn, layers=len(self.layers), rms_eps=self.eps,
                        final_norm=1 if self.apply_final_norm else 0, use_graph=1 if self.use_graph else 0,
                        no_qk_norm=0 if self.qk_norm else 1, norm_weight_first=1 if self.norm_weight_first else 0,
                        causal_block=self.causal_block)
        arr = (LlmLayerWeights * len(self.layers))()
        for i, layer in enumerate(self.layers):
            a, m = layer.self_attn, layer.mlp
            qn = self._bf16(a.q_norm.weight) if self.qk_norm else None
            kn = self._bf16(a.k_norm.weight) if self.qk_norm else None
            arr[i] = LlmLayerWeights(
                self._bf16(layer.input_layernorm.weight), self._bf16(a.q_proj.weight), self._bf16(a.k_proj.weight),
                self._bf16(a.v_proj.weight), qn, kn,
                self._bf16(a.o_proj.weight), self._bf16(layer.post_attention_layernorm.weight),
                self._bf16(m.gate_proj.weight), self._bf16(m.up_proj.weight), self._bf16(m.down_proj.weight))
        w = LlmWeights(C.cast(arr, C.POINTER(LlmLayerWeights)),
                       self._bf16(self.norm.weight) if self.apply_final_norm else None,
                       self.cos.data_ptr(), self.sin.data_ptr())
        handle = C.c_void_p()
        with torch.cuda.device(self.device):
            rc = _lib.load().rldx_llm_create(C.byref(cfg), C.byref(w), C.byref(handle))
        self._keep.clear()  # the runtime copied every weight into its own arena
        check(rc)
        self._handle = handle
        self._batch = batch

    @property
    def launches_per_call(self) -> int:
        return int(_lib.load().rldx_llm_launch_count(self._handle)) if self._handle else 0

    def forward(self, hidden_states: torch.Tensor, deepstack_features=None,
                deepstack_flat_indices=None) -> torch.Tensor:
        if deepstack_features is not None:
            raise NotImplementedError("deepstack feature injection is not bound")
        if hidden_states.dim() == 2:
            hidden_states = hidden_states.unsqueeze(0)
        B, M, D = hidden_states.shape
        if M != self.cos.shape[0] or D != self.hidden:
            raise ValueError(f"hidden_states {tuple(hidden_states.shape)} does not match the chain's "
                             f"[*, {self.cos.shape[0]}, {self.hidden}]")
        if self._handle is None:
            self.bind(B)
        elif B != self._batch:
            raise ValueError(f"batch {B} differs from the bound batch {self._batch}")
        x = hidden_states
        if x.device != self.device or x.dtype != torch.bfloat16 or not x.is_contiguous():
            x = x.to(device=self.device, dtype=torch.bfloat16).contiguous()
        out = torch.empty_like(x)
        stream = torch.cuda.current_stream(self.device)
        check(_lib.load().rldx_llm_prefill(self._handle, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                           C.c_void_p(stream.cuda_stream)))
        return out

    def __del__(self):
        h = self.__dict__.pop("_handle", None)
        if h:
            try:
                _lib.load().rldx_llm_destroy(h)
            except Exception:  # noqa: BLE001
                pass


class B200MemoryChain(nn.Module):
    """Drop-in for CustomMemoryChain (rldx/inference/memory/engine/custom_memory_chain.py:43-174):

        chain = B200MemoryChain(gs_memory, device)      # GraphSafeMemory or TransformerMemory
        out = chain(inputs_embeds)                       # [B, M, D] -> [B, M, D]

    TransformerMemory (rldx/model/modules/memory.py:230-370): RoPE-only attention (no q / k
    norm) with block-wise positions token // block_attn_size, the token-causal mask
    (use_causal_attn) or the block mask, weight-then-cast RMSNorm, final norm.  Native runtime:
    the decoder-stack path of librldx_b200 (96-dim heads run zero-padded to 128)."""

    def __init__(self, gs_memory, device=None, dtype=torch.bfloat16, *, use_graph: bool = True):
        super().__init__()
        if dtype != torch.bfloat16:
            raise ValueError("the B200 memory chain computes in bfloat16 only")
        self.memory = getattr(gs_memory, "_memory", gs_memory)
        self.static_position_ids = getattr(gs_memory, "static_position_ids", None)
        m = self.memory
        cfg = getattr(m, "c", None)
        self.block = int(getattr(m, "block_attn_size", getattr(cfg, "block", 1)))
        self.use_causal_attn = bool(getattr(m, "use_causal_attn", getattr(cfg, "use_causal_attn", True)))
        if not getattr(m, "use_rope", True):
            raise NotImplementedError("TransformerMemory(use_rope=False) (sinusoidal positions) is not bound")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.use_graph = use_graph
        self._chain = None
        self._tokens = None

    def _tables(self, M: int):
        attn = self.memory.layers[0].self_attn
        if self.static_position_ids is not None:
            pos = self.static_position_ids.reshape(-1)[:M].float().cpu()
        else:
            pos = (torch.arange(M) // self.block).float()
        inv = attn.rotary_emb.inv_freq.detach().float().cpu()
        freqs = pos[:, None] * inv[None, :]
        emb = torch.cat([freqs, freqs], dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        ssin = sin.clone()
        ssin[:, : ssin.shape[-1] // 2] *= -1
        return cos, ssin

    def forward(self, inputs_embeds: torch.Tensor) -> torch.Tensor:
        M = inputs_embeds.shape[-2]
        if self._chain is None:
            cos, ssin = self._tables(M)
            self._chain = B200LLMChain(self.memory.layers, self.memory.norm, cos.to(self.device), ssin.to(self.device),
                                       apply_final_norm=True, device=self.device, use_graph=self.use_graph,
                                       norm_weight_first=True,
                                       causal_block=1 if self.use_causal_attn else self.block)
            self._tokens = M
        elif M != self._tokens:
            raise ValueError(f"{M} tokens differ from the bound {self._tokens}")
        return self._chain(inputs_embeds)
