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
then runs as one CUDA graph of hand-written sm_100a kernels.  Deepstack features
(`deepstack_features[i]` [n, hidden] with `deepstack_flat_indices`, the element indices of the
n visual token rows in one [tokens, hidden] sequence, as CustomLLMChain takes them,
custom_llm_chain.py:137-161) are added after layer i to those rows of every sequence, with the
eager path's single bf16 rounding (Qwen3VLTextModel._deepstack_process,
modeling_qwen3_vl.py:1102-1113); the rows and the number of deepstack layers are bound on the
first call.

Video-token compression (the VTC backbone wraps every text layer in LayerWrapper with
internal_projection=4, rldx/model/modules/backbone/modeling_vtc.py:158-164) runs inside the same
graph: `compress_info` (the dict of the reference's _find_compress_info,
rldx/inference/backbone/llm/model/graph_safe_qwen3vl_text_model.py:26-59, which
find_compress_info below computes from the prompt's input_ids) makes the chain replace the old
frames' token rows [static_begin, static_end) with their mean before layer compress_layer_idx;
the output then has static_out_len tokens.  Where the reference engine runs a pre-compression
chain, a torch compress step and a post-compression chain (custom_backbone_chain.py:177-214),
this is one chain and one graph.
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


def find_compress_rows(input_ids: torch.Tensor, img_pattern=(151652,), num_views=None):
    """Static (begin, end) of the compressed region, the rows LayerWrapper.get_removing_indices
    finds (layer_wrapper.py:25-51): begin = the first occurrence of `img_pattern` (the image-start
    marker), end = its last occurrence, or the num_views-th last with image-wise encoding.  The
    reference engine takes sequence 0's rows for the whole batch; here every sequence must give
    the same rows (a batch whose prompts differ would be compressed wrongly), else ValueError."""
    ids = input_ids.detach().to("cpu", torch.int64)
    if ids.dim() == 1:
        ids = ids[None]
    pat = torch.as_tensor(list(img_pattern), dtype=torch.int64)
    n = pat.numel()
    if ids.shape[1] < n:
        raise ValueError("input_ids shorter than the image pattern")
    hit = torch.ones(ids.shape[0], ids.shape[1] - n + 1, dtype=torch.bool)
    for j in range(n):
        hit &= ids[:, j: ids.shape[1] - n + 1 + j] == pat[j]
    rows = set()
    for b in range(ids.shape[0]):
        pos = torch.nonzero(hit[b]).flatten().tolist()
        if not pos:
            raise ValueError(f"sequence {b} has no image-start marker {list(img_pattern)}")
        if num_views is not None and int(num_views) > len(pos):
            raise ValueError(f"sequence {b} has {len(pos)} markers, fewer than num_views={num_views}")
        rows.add((pos[0], pos[-int(num_views)] if num_views is not None else pos[-1]))
    if len(rows) != 1:
        raise ValueError(f"the sequences of the batch compress different rows: {sorted(rows)}")
    return rows.pop()


def find_compress_info(layers, input_ids: torch.Tensor, n_cog_tokens: int = 0, num_views=None):
    """The reference's _find_compress_info (graph_safe_qwen3vl_text_model.py:26-59): the first
    LayerWrapper whose layer_idx equals its internal_projection compresses; returns
    {"compress_layer_idx", "static_begin", "static_end", "static_out_len"}, or None when no layer
    compresses or begin >= end (one frame: LayerWrapper's compress_mask is false)."""
    for idx, layer in enumerate(layers):
        if hasattr(layer, "layer") and hasattr(layer, "internal_projection") and \
                layer.layer_idx == layer.internal_projection:
            b, e = find_compress_rows(input_ids, getattr(layer, "img_pattern", (151652,)), num_views)
            if b >= e:
                return None
            L = int(input_ids.shape[-1]) + int(n_cog_tokens)
            return {"compress_layer_idx": idx, "static_begin": b, "static_end": e, "static_out_len": b + 1 + (L - e)}
    return None


def unsigned_sin(signed_sin: torch.Tensor) -> torch.Tensor:
    half = signed_sin.shape[-1] // 2
    sin = signed_sin.clone()
    sin[..., :half] = -sin[..., :half]
    return sin


class B200LLMChain(nn.Module):
    """norm_weight_first / causal_block select the memory module's variant (see
    B200MemoryChain); a layer without q_norm / k_norm runs without the per-head QK RMSNorm.
    compress_info: video-token compression (find_compress_info's dict); pos_cos / signed_sin are
    then the tables of the uncompressed sequence."""

    def __init__(self, layers, norm: nn.Module, pos_cos: torch.Tensor, signed_sin: torch.Tensor,
                 apply_final_norm: bool = True, *, device=None, use_graph: bool = True,
                 norm_weight_first: bool = False, causal_block: int = 1, compress_info: Optional[dict] = None):
        super().__init__()
        self.compress_info = dict(compress_info) if compress_info else None
        if self.compress_info is not None:
            ci = self.compress_info
            M = pos_cos.shape[0]
            b, e, li = int(ci["static_begin"]), int(ci["static_end"]), int(ci["compress_layer_idx"])
            if not (0 <= b < e <= M and 0 <= li < len(layers)):
                raise ValueError(f"compress_info {ci} does not fit {len(layers)} layers over {M} tokens")
            if "static_out_len" in ci and int(ci["static_out_len"]) != M - (e - b) + 1:
                raise ValueError(f"compress_info static_out_len {ci['static_out_len']} != {M - (e - b) + 1}")
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
        self._ds = None  # (layers, rows) bound at create

    def _bf16(self, t: torch.Tensor) -> int:
        t = t.detach().to(device=self.device, dtype=torch.bfloat16).contiguous()
        self._keep.append(t)
        return t.data_ptr()

    def bind(self, batch: int, deepstack_rows: Optional[torch.Tensor] = None, deepstack_layers: int = 0) -> None:
        M = self.cos.shape[0]
        nrows = 0 if deepstack_rows is None else int(deepstack_rows.numel())
        cfg = LlmConfig(batch=batch, tokens=M, hidden=self.hidden, q_heads=self.q_heads, kv_heads=self.kv_heads,
                        head_dim=self.head_dim, ffn=self.ffn, layers=len(self.layers), rms_eps=self.eps,
                        final_norm=1 if self.apply_final_norm else 0, use_graph=1 if self.use_graph else 0,
                        no_qk_norm=0 if self.qk_norm else 1, norm_weight_first=1 if self.norm_weight_first else 0,
                        causal_block=self.causal_block, deepstack_layers=deepstack_layers if nrows else 0,
                        deepstack_rows=nrows)
        if self.compress_info is not None:
            cfg.compress_layer = int(self.compress_info["compress_layer_idx"])
            cfg.compress_begin = int(self.compress_info["static_begin"])
            cfg.compress_end = int(self.compress_info["static_end"])
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
        rows_c = None
        if nrows:
            rows_c = (C.c_int * nrows)(*[int(r) for r in deepstack_rows.tolist()])
        w = LlmWeights(C.cast(arr, C.POINTER(LlmLayerWeights)),
                       self._bf16(self.norm.weight) if self.apply_final_norm else None,
                       self.cos.data_ptr(), self.sin.data_ptr(),
                       C.cast(rows_c, C.POINTER(C.c_int)) if rows_c is not None else None)
        handle = C.c_void_p()
        with torch.cuda.device(self.device):
            rc = _lib.load().rldx_llm_create(C.byref(cfg), C.byref(w), C.byref(handle))
        self._keep.clear()  # the runtime copied every weight into its own arena
        check(rc)
        self._handle = handle
        self._batch = batch
        self._ds = (deepstack_layers, tuple(deepstack_rows.tolist())) if nrows else None

    @property
    def out_tokens(self) -> int:
        """Tokens per sequence of the output (the compressed count with compress_info)."""
        if self._handle:
            return int(_lib.load().rldx_llm_out_tokens(self._handle))
        M = self.cos.shape[0]
        ci = self.compress_info
        return M - (int(ci["static_end"]) - int(ci["static_begin"])) + 1 if ci else M

    @property
    def launches_per_call(self) -> int:
        return int(_lib.load().rldx_llm_launch_count(self._handle)) if self._handle else 0

    def _deepstack_rows(self, deepstack_flat_indices: torch.Tensor) -> torch.Tensor:
        """Token rows of the reference's flat element indices (row * hidden + column, whole rows)."""
        flat = deepstack_flat_indices.detach().reshape(-1).to("cpu", torch.int64)
        D = self.hidden
        if flat.numel() == 0 or flat.numel() % D:
            raise ValueError("deepstack_flat_indices must cover whole rows of the hidden width")
        rows = flat.view(-1, D)[:, 0] // D
        if not torch.equal(flat.view(-1, D), rows[:, None] * D + torch.arange(D)[None, :]):
            raise NotImplementedError("deepstack_flat_indices must list whole rows, columns in order")
        return rows

    def forward(self, hidden_states: torch.Tensor, deepstack_features=None,
                deepstack_flat_indices=None) -> torch.Tensor:
        if hidden_states.dim() == 2:
            hidden_states = hidden_states.unsqueeze(0)
        B, M, D = hidden_states.shape
        if M != self.cos.shape[0] or D != self.hidden:
            raise ValueError(f"hidden_states {tuple(hidden_states.shape)} does not match the chain's "
                             f"[*, {self.cos.shape[0]}, {self.hidden}]")
        ds = None
        if deepstack_features is not None and len(deepstack_features) > 0:
            if deepstack_flat_indices is None:
                raise ValueError("deepstack_features need deepstack_flat_indices")
            ds = (min(len(deepstack_features), len(self.layers)), self._deepstack_rows(deepstack_flat_indices))
        if self._handle is None:
            self.bind(B, ds[1] if ds else None, ds[0] if ds else 0)
        elif B != self._batch:
            raise ValueError(f"batch {B} differs from the bound batch {self._batch}")
        if (ds is None) != (self._ds is None) or (ds is not None and (ds[0], tuple(ds[1].tolist())) != self._ds):
            raise ValueError("deepstack layers / rows differ from the ones bound on the first call")
        x = hidden_states
        if x.device != self.device or x.dtype != torch.bfloat16 or not x.is_contiguous():
            x = x.to(device=self.device, dtype=torch.bfloat16).contiguous()
        out = torch.empty(B, self.out_tokens, D, dtype=torch.bfloat16, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        if ds is not None:
            L, rows = ds
            n = rows.numel()
            feats = torch.stack([deepstack_features[i].reshape(n, D) for i in range(L)])
            # every sequence gets the same features (the reference chain's [1, tokens, hidden] buffer)
            feats = feats.to(device=self.device, dtype=torch.bfloat16)[:, None].expand(L, B, n, D).contiguous()
            check(_lib.load().rldx_llm_set_deepstack(self._handle, C.c_void_p(feats.data_ptr()),
                                                     C.c_void_p(stream.cuda_stream)))
            self._keep_ds = feats  # alive until the copy queued on `stream` has run
        code = self.device_status(wait=False)  # an error recorded by an earlier asynchronous call
        if code:
            raise _lib.RldxError(_lib.RLDX_ERR_DEVICE, f"device error 0x{code:x} recorded by a prefill")
        check(_lib.load().rldx_llm_prefill(self._handle, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                           C.c_void_p(stream.cuda_stream)))
        return out

    def device_status(self, wait: bool = True) -> int:
        """Device error code of the last prefill (0: none; with wait=False, 0 while it is still
        running).  Reading clears it."""
        if self._handle is None:
            return 0
        code = C.c_uint(0)
        check(_lib.load().rldx_llm_status(self._handle, 1 if wait else 0, C.byref(code)))
        return int(code.value)

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


class B200MemoryCache(nn.Module):
    """The recurrent memory of the VLA on the native memory chain: the counterpart of
    GraphSafeVLA's memory state and _process_memory (rldx/inference/model/graph_safe_vla.py:38-68,
    106-140):

        mem = B200MemoryCache(gs_memory, memory_config, batch=B, device="cuda:0")
        vl = mem(vl_embs)          # [B, n_q, d] backbone cognition tokens -> decoder VL tokens
        mem.reset_memory()         # new episode: the cached sets go back to zeros

    Each call shifts the cache of the last `memory_length` sets of `memory_n_cog_tokens` tokens
    by one set, appends the current set (the last memory_n_cog_tokens of the n_cog_tokens
    cognition tokens), runs TransformerMemory over the cache (B200MemoryChain) and returns the
    cognition tokens followed by the memory output of the newest set (concat_memory), or the
    passed-through tokens followed by it.  One cache per sequence of the batch (the reference
    keeps one, batch 1); the cache lives on the device and is updated in place."""

    def __init__(self, gs_memory, memory_config: dict, batch: int = 1, device=None, *, use_graph: bool = True):
        super().__init__()
        self.n_q = int(memory_config["n_cog_tokens"])
        self.n_cog_mem = int(memory_config["memory_n_cog_tokens"])
        self.n_cog_pass = self.n_q - self.n_cog_mem
        self.memory_length = int(memory_config["memory_length"])
        self.concat_memory = bool(memory_config["concat_memory"])
        d = int(memory_config["hidden_size"])
        self.chain = B200MemoryChain(gs_memory, device, use_graph=use_graph)
        self.device = self.chain.device
        K, n = self.memory_length, self.n_cog_mem
        self._cached_cog = torch.zeros(batch, K * n, d, dtype=torch.bfloat16, device=self.device)
        self._cache_tmp = torch.zeros_like(self._cached_cog)

    def reset_memory(self) -> None:
        self._cached_cog.zero_()

    def forward(self, vl_embs: torch.Tensor) -> torch.Tensor:
        if vl_embs.shape[0] != self._cached_cog.shape[0] or vl_embs.shape[-1] != self._cached_cog.shape[-1]:
            raise ValueError(f"vl_embs {tuple(vl_embs.shape)} does not match the cache "
                             f"[{self._cached_cog.shape[0]}, *, {self._cached_cog.shape[-1]}]")
        cog_all = vl_embs[:, -self.n_q:, :]
        cog_current = cog_all[:, self.n_cog_pass:, :]
        n = self.n_cog_mem
        self._cache_tmp[:, :-n, :].copy_(self._cached_cog[:, n:, :])
        self._cache_tmp[:, -n:, :].copy_(cog_current)
        self._cached_cog.copy_(self._cache_tmp)
        memory_out = self.chain(self._cached_cog)
        cog_augmented = memory_out[:, -n:, :]
        if self.concat_memory:
            return torch.cat([cog_all.to(cog_augmented.dtype), cog_augmented], dim=1)
        if self.n_cog_pass > 0:
            return torch.cat([cog_all[:, : self.n_cog_pass, :].to(cog_augmented.dtype), cog_augmented], dim=1)
        return cog_augmented
