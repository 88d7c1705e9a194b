"""ctypes binding of librldx_b200.so: structures mirror include/rldx_b200.h field for field.

Loading fails loudly (ImportError / RuntimeError) when the library is missing: there is no
fallback implementation anywhere in this package.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "librldx_b200.so"

RLDX_OK = 0
RLDX_ERR_ARG = -1
RLDX_ERR_CUDA = -2
RLDX_ERR_DEVICE = -3
RLDX_ERR_UNSUPPORTED = -4
RLDX_ERR_STATE = -5

EPI_STORE, EPI_SWIGLU, EPI_QKV, EPI_EULER = 0, 1, 2, 3
BIAS_NONE, BIAS_FUSED, BIAS_POST_ROUND = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_SILU, ACT_SWISH = 0, 1, 2, 3
ROPE_SA_ONLY, ROPE_VL_SA = 0, 1

vp = C.c_void_p
i64 = C.c_int64


class GemmDesc(C.Structure):
    _fields_ = [
        ("a", vp), ("lda", i64),
        ("b", vp), ("ldb", i64), ("b_cat_stride", i64),
        ("cat_ids", vp), ("rows_per_cat", C.c_int), ("num_cats", C.c_int),
        ("M", C.c_int), ("N", C.c_int), ("K", C.c_int),
        ("bias", vp), ("bias_mode", C.c_int), ("bias_cat_stride", i64), ("act", C.c_int),
        ("add", vp), ("ld_add", i64), ("add_row_mod", C.c_int),
        ("out", vp), ("ldo", i64), ("col_off", C.c_int),
        ("epilogue", C.c_int),
        ("rows_in", C.c_int), ("rows_out", C.c_int), ("row_skip", C.c_int),
        ("dt", C.c_float),
        ("q_norm_w", vp), ("k_norm_w", vp), ("rope_cos", vp), ("rope_sin", vp),
        ("q", vp), ("k", vp), ("vt", vp),
        ("L", C.c_int), ("Lp", C.c_int), ("H", C.c_int), ("tok_off", C.c_int),
        ("eps", C.c_float),
        ("tile_n", C.c_int), ("rope_identity", C.c_int),
    ]


class MsatConfig(C.Structure):
    _fields_ = [
        ("batch", C.c_int), ("n_vl", C.c_int), ("n_state", C.c_int), ("horizon", C.c_int),
        ("physics_hist", C.c_int), ("physics_fut", C.c_int), ("dim", C.c_int),
        ("heads", C.c_int), ("head_dim", C.c_int), ("depth", C.c_int),
        ("mlp_hidden", C.c_int), ("vl_mlp_hidden", C.c_int), ("out_dim", C.c_int),
        ("action_dim", C.c_int), ("state_dim", C.c_int), ("dec_hidden", C.c_int),
        ("physics_dim", C.c_int), ("num_embodiments", C.c_int), ("num_steps", C.c_int),
        ("rope_mode", C.c_int), ("rope_cos_only", C.c_int), ("rope_theta", C.c_float),
        ("rope_max_seq", C.c_int), ("temb_channels", C.c_int), ("use_graph", C.c_int),
        ("standard_path", C.c_int), ("vl_dim", C.c_int), ("depth_single", C.c_int),
        ("single_expanded", C.c_int), ("single_mlp_hidden", C.c_int), ("prefix_len", C.c_int),
        ("key_mask", C.c_int),
    ]


class Linear(C.Structure):
    _fields_ = [("w", vp), ("b", vp)]


class CatLinear(C.Structure):
    _fields_ = [("W", vp), ("b", vp)]


class StreamWeights(C.Structure):
    _fields_ = [("qkv", Linear), ("proj", Linear), ("w12", Linear), ("w3", Linear),
                ("q_norm", vp), ("k_norm", vp)]


class BlockWeights(C.Structure):
    _fields_ = [("vl", StreamWeights), ("sa", StreamWeights), ("p", StreamWeights)]


class SingleBlockWeights(C.Structure):
    _fields_ = [("linear1", Linear), ("linear2", Linear), ("mlp_proj", Linear),
                ("q_norm", vp), ("k_norm", vp),
                ("p_linear1", Linear), ("p_linear2", Linear), ("p_mlp_proj", Linear),
                ("p_q_norm", vp), ("p_k_norm", vp)]


class MsatWeights(C.Structure):
    _fields_ = [
        ("blocks", C.POINTER(BlockWeights)),
        ("temb_lin1", Linear), ("temb_lin2", Linear), ("time_token_proj", Linear),
        ("proj_out_1", Linear), ("proj_out_2", Linear),
        ("proj_out_phys_1", Linear), ("proj_out_phys_2", Linear),
        ("state_l1", CatLinear), ("state_l2", CatLinear),
        ("act_w1", CatLinear), ("act_w2", CatLinear), ("act_w3", CatLinear),
        ("dec_l1", CatLinear), ("dec_l2", CatLinear),
        ("pos_emb", vp),
        ("phc_w1", Linear), ("phc_w2", Linear), ("phc_w3", Linear),
        ("phf_w1", Linear), ("phf_w2", Linear), ("phf_w3", Linear),
        ("phd_l1", Linear), ("phd_l2", Linear),
        ("single_blocks", C.POINTER(SingleBlockWeights)), ("vl_proj_to_sa", Linear),
        ("rope_cos", vp * 2), ("rope_sin", vp * 2),
    ]


class OpProfile(C.Structure):
    _fields_ = [("kind", C.c_int), ("grid", C.c_int), ("ms", C.c_float), ("bytes", C.c_double),
                ("flops", C.c_double)]


class AttentionDesc(C.Structure):
    _fields_ = [("q", vp), ("k", vp), ("vt", vp), ("B", C.c_int), ("H", C.c_int),
                ("kv_heads", C.c_int), ("L", C.c_int), ("Lp", C.c_int), ("head_dim", C.c_int),
                ("causal", C.c_int), ("tiles_per_cta", C.c_int), ("key_mask", vp),
                ("out", vp * 3), ("seg_len", C.c_int * 3), ("out_ld", C.c_int * 3), ("nseg", C.c_int),
                ("causal_block", C.c_int), ("out_dim", C.c_int)]


class QkvSegment(C.Structure):
    _fields_ = [("qkv", vp), ("ld", i64), ("batch_stride", i64), ("rows", C.c_int),
                ("rope_from", C.c_int), ("q_norm", vp), ("k_norm", vp), ("rope_cos", vp),
                ("rope_sin", vp)]


class ResLnSegment(C.Structure):
    _fields_ = [("x", vp), ("y", vp), ("v1", vp), ("v2", vp), ("sum_out", vp), ("ln_out", vp),
                ("rows", C.c_int), ("D", C.c_int), ("ld", i64), ("w", vp)]


class SwigluBiasSegment(C.Structure):
    _fields_ = [("gate", vp), ("up", vp), ("bias_gate", vp), ("bias_up", vp), ("out", vp),
                ("ld_in", i64), ("ld_out", i64), ("rows", C.c_int), ("H", C.c_int)]


class LlmConfig(C.Structure):
    _fields_ = [("batch", C.c_int), ("tokens", C.c_int), ("hidden", C.c_int), ("q_heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn", C.c_int), ("layers", C.c_int),
                ("rms_eps", C.c_float), ("final_norm", C.c_int), ("use_graph", C.c_int),
                ("no_qk_norm", C.c_int), ("norm_weight_first", C.c_int), ("causal_block", C.c_int),
                ("deepstack_layers", C.c_int), ("deepstack_rows", C.c_int), ("compress_layer", C.c_int),
                ("compress_begin", C.c_int), ("compress_end", C.c_int)]


class LlmLayerWeights(C.Structure):
    _fields_ = [(n, vp) for n in ("input_norm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
                                  "post_norm", "gate_proj", "up_proj", "down_proj")]


class LlmWeights(C.Structure):
    _fields_ = [("layers", C.POINTER(LlmLayerWeights)), ("final_norm", vp), ("rope_cos", vp),
                ("rope_sin", vp), ("deepstack_row_index", C.POINTER(C.c_int))]


class MsatIO(C.Structure):
    _fields_ = [("vl", vp), ("state", vp), ("emb_id", vp), ("init_noise", vp),
                ("physics_hist", vp), ("physics_noise", vp), ("actions", vp),
                ("prefix_actions", vp), ("vl_mask", vp), ("physics_mask", vp)]


# Every exported symbol of include/rldx_b200.h with its ctypes signature.
SIGNATURES = {
    "rldx_version": (C.c_int, []),
    "rldx_last_error": (C.c_char_p, []),
    "rldx_get_device_error": (C.c_int, [C.POINTER(C.c_uint)]),
    "rldx_device_supported": (C.c_int, []),
    "rldx_gemm": (C.c_int, [C.POINTER(GemmDesc), C.c_int, vp]),
    "rldx_gemm_workspace_size": (C.c_int, [C.POINTER(GemmDesc), C.c_int, C.POINTER(C.c_uint64)]),
    "rldx_gemm_plan": (C.c_int, [C.POINTER(GemmDesc), C.c_int, C.POINTER(C.c_int)]),
    "rldx_gemm_ws": (C.c_int, [C.POINTER(GemmDesc), C.c_int, vp, C.c_uint64, vp]),
    "rldx_gemm_static_ws": (C.c_int, [C.POINTER(GemmDesc), C.c_int, vp]),
    "rldx_joint_attention": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp,
                                       C.POINTER(vp), C.POINTER(C.c_int), C.c_int, C.c_int, vp]),
    "rldx_layernorm": (C.c_int, [vp, i64, vp, i64, C.c_int, C.c_int, C.c_float, vp, vp, vp]),
    "rldx_attention": (C.c_int, [C.POINTER(AttentionDesc), vp]),
    "rldx_llm_create": (C.c_int, [C.POINTER(LlmConfig), C.POINTER(LlmWeights), C.POINTER(vp)]),
    "rldx_llm_destroy": (C.c_int, [vp]),
    "rldx_llm_prefill": (C.c_int, [vp, vp, vp, vp]),
    "rldx_llm_launch_count": (C.c_int, [vp]),
    "rldx_llm_out_tokens": (C.c_int, [vp]),
    "rldx_llm_set_deepstack": (C.c_int, [vp, vp, vp]),
    "rldx_qkv_prep": (C.c_int, [C.POINTER(QkvSegment), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_float, vp, vp, vp, vp]),
    "rldx_res_layernorm": (C.c_int, [C.POINTER(ResLnSegment), C.c_int, C.c_int, C.c_float, vp]),
    "rldx_res_rmsnorm": (C.c_int, [C.POINTER(ResLnSegment), C.c_int, C.c_float, vp]),
    "rldx_swiglu_bias": (C.c_int, [C.POINTER(SwigluBiasSegment), C.c_int, vp]),
    "rldx_qk_rmsnorm_rope": (C.c_int, [vp, vp, vp, vp, vp, vp, i64, C.c_int, C.c_int,
                                       C.c_float, vp]),
    "rldx_swiglu": (C.c_int, [vp, vp, i64, vp, i64, i64, C.c_int, vp]),
    "rldx_msat_create": (C.c_int, [C.POINTER(MsatConfig), C.POINTER(MsatWeights), C.POINTER(vp)]),
    "rldx_msat_destroy": (C.c_int, [vp]),
    "rldx_msat_step": (C.c_int, [vp, C.POINTER(MsatIO), vp]),
    "rldx_msat_step_host": (C.c_int, [vp, C.POINTER(MsatIO), vp]),
    "rldx_msat_launch_count": (C.c_int, [vp]),
    "rldx_msat_profile": (C.c_int, [vp, C.POINTER(MsatIO), C.POINTER(OpProfile), C.c_int,
                                    C.POINTER(C.c_int), vp]),
    "rldx_msat_read_buffer": (C.c_int, [vp, C.c_int, vp, i64, C.POINTER(i64), C.POINTER(i64),
                                        vp]),
    "rldx_msat_status": (C.c_int, [vp, C.c_int, C.POINTER(C.c_uint)]),
    "rldx_msat_block_end": (C.c_int, [vp, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "rldx_msat_run_partial": (C.c_int, [vp, C.POINTER(MsatIO), C.c_int, vp]),
    "rldx_llm_status": (C.c_int, [vp, C.c_int, C.POINTER(C.c_uint)]),
    "rldx_set_wait_limit": (C.c_int, [i64]),
    "rldx_get_wait_limit": (C.c_int, [C.POINTER(i64)]),
    "rldx_wait_selftest": (C.c_int, [i64, vp]),
}

_LIB = None


def load(path: Path | None = None) -> C.CDLL:
    """Loads the library once (building it first when sources are newer)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    lib_path = Path(path) if path else LIB_PATH
    if path is None:
        from . import build as _build  # noqa: PLC0415

        if _build.needs_build():
            _build.build()
    if not lib_path.exists():
        raise ImportError(f"{lib_path} not found: build it with `python -m rldx_b200.build`")
    lib = C.CDLL(str(lib_path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class RldxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rldx error {code}: {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != RLDX_OK:
        msg = load().rldx_last_error()
        raise RldxError(rc, msg.decode() if msg else "")
