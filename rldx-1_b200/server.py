"""Server compile levels: the reference server's `--compile` switch with a level for this library.

The reference inference server maps its `--compile` levels to optimization paths and applies
the chosen path after loading the policy (rldx/eval/run_rldx_server.py:103-126, 148-197):

    _COMPILE_LEVEL_TO_PATH = {"none": "A", "submodule": "B", "fullgraph": "D"}

This module keeps those three levels and adds `b200`, which installs the native action head
(`serve.apply_optimization(policy, "B200")`: the B200 chain behind `model.get_action`).  The
reference's own levels are delegated to the reference's `apply_optimization` when it is
importable; the B200 level needs only this package.

    level = parse_compile_level(args.compile)          # "none" | "submodule" | "fullgraph" | "b200"
    validate_compile_level(level, rtc_inference_mode)  # before the model load, as _validate_cli
    info = apply_compile_level(policy, level)          # after the policy is loaded
"""

from __future__ import annotations

from typing import Any, Optional

from . import serve

# the reference's levels (run_rldx_server.py:117) and the native one
COMPILE_LEVEL_TO_PATH = {"none": "A", "submodule": "B", "fullgraph": "D", "b200": "B200"}


def parse_compile_level(level: Optional[str]) -> Optional[str]:
    """The path letter of a --compile level (None for eager, as _resolve_compile_level)."""
    if level is None:
        return None
    key = str(level).lower()
    if key not in COMPILE_LEVEL_TO_PATH:
        raise ValueError(f"unknown --compile level {level!r}; expected one of {sorted(COMPILE_LEVEL_TO_PATH)}")
    path = COMPILE_LEVEL_TO_PATH[key]
    return None if path == "A" else path


def validate_compile_level(level: Optional[str], rtc_inference_mode: Optional[str]) -> Optional[str]:
    """Rejects the combinations the reference rejects before loading the model
    (run_rldx_server.py:128-139): a compiled whole-chain path (D, and B200, which captures the
    whole control step in one CUDA graph) cannot route the VJP of RTC `guided` mode."""
    path = parse_compile_level(level)
    if path in {"C", "D", "B200"} and rtc_inference_mode == "guided":
        raise ValueError(f"--compile={level} is incompatible with --rtc-inference-mode=guided: the "
                         "captured control step cannot route a VJP through action_prefix; use "
                         "--compile=submodule or --rtc-inference-mode in {none, trained}")
    return path


def apply_compile_level(policy: Any, level: Optional[str], **kwargs) -> Optional[dict]:
    """Applies a --compile level to a loaded policy; returns the installer's info (None: eager)."""
    path = parse_compile_level(level)
    if path is None:
        return None
    if path == "B200":
        return serve.apply_optimization(policy, "B200", **kwargs)
    try:  # the reference's own torch.compile paths
        from rldx.inference.serve_optimization import apply_optimization as reference_apply
    except ImportError as e:
        raise RuntimeError(f"--compile={level} is the reference's path {path}: it needs the reference "
                           "package (rldx.inference.serve_optimization)") from e
    return reference_apply(policy, path=path)
