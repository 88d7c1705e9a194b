"""C-ABI surface (CPU only): the library loads and exports every function that
include/rldx_b200.h declares, and the ctypes mirrors match the header's structs."""

import ctypes as C
import re
from pathlib import Path

import rldx_b200  # noqa: F401
from rldx_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "rldx_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(rldx_\w+)\s*\(", text, flags=re.M)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in rldx_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_error_string(lib):
    assert lib.rldx_version() == 111
    assert isinstance(lib.rldx_last_error(), bytes)


def test_struct_layouts_match_header():
    # sizes of the C structs as laid out by the C compiler on this ABI (x86-64 / aarch64 LP64)
    assert C.sizeof(_lib.GemmDesc) == 256
    assert C.sizeof(_lib.MsatConfig) == 32 * 4
    assert C.sizeof(_lib.MsatIO) == 10 * 8
    assert C.sizeof(_lib.BlockWeights) == 3 * (4 * 16 + 16)
    assert C.sizeof(_lib.SingleBlockWeights) == 2 * (3 * 16 + 16)
    assert C.sizeof(_lib.QkvSegment) == 64
    assert C.sizeof(_lib.LlmConfig) == 19 * 4 and C.sizeof(_lib.LlmLayerWeights) == 11 * 8
    assert C.sizeof(_lib.LlmWeights) == 5 * 8
    assert C.sizeof(_lib.AttentionDesc) == 3 * 8 + 8 * 4 + 8 + 3 * 8 + 3 * 4 + 3 * 4 + 3 * 4 + 4
    assert C.sizeof(_lib.ResLnSegment) == 6 * 8 + 2 * 4 + 8 + 8
    assert C.sizeof(_lib.SwigluBiasSegment) == 5 * 8 + 2 * 8 + 2 * 4


def test_null_arguments_are_rejected_without_a_device(lib):
    # argument validation happens before any device work
    assert lib.rldx_get_device_error(None) == _lib.RLDX_ERR_ARG
    assert lib.rldx_msat_step(None, None, None) == _lib.RLDX_ERR_ARG
    assert lib.rldx_msat_create(None, None, None) == _lib.RLDX_ERR_ARG
    assert lib.rldx_msat_destroy(None) == _lib.RLDX_OK
    code = C.c_uint(7)
    assert lib.rldx_msat_status(None, 1, C.byref(code)) == _lib.RLDX_ERR_ARG
    assert lib.rldx_llm_status(None, 1, C.byref(code)) == _lib.RLDX_ERR_ARG
    n = C.c_int(0)
    assert lib.rldx_msat_block_end(None, 0, 0, C.byref(n)) == _lib.RLDX_ERR_ARG
    assert lib.rldx_msat_run_partial(None, None, 0, None) == _lib.RLDX_ERR_ARG
    assert lib.rldx_get_wait_limit(None) == _lib.RLDX_ERR_ARG
    assert lib.rldx_llm_out_tokens(None) == 0 and lib.rldx_llm_launch_count(None) == 0
