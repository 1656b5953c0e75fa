"""The C-ABI library loads without a GPU and exports every declared symbol. CPU only."""

from __future__ import annotations

import ctypes
import os
import re

import deepseek_v41_mlx_b200 as q
from deepseek_v41_mlx_b200 import _lib as L

from conftest import ROOT


def _header_functions():
    src = open(os.path.join(ROOT, "include", "dsv41q.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dsv41_[a-z0-9_]+)\s*\(", src)))


def test_library_built_and_loads():
    assert os.path.exists(q.lib_path()), "run deepseek-v41-mlx_b200/build.py"
    lib = L.load()
    assert lib.dsv41_abi_version() == 1


def test_every_header_symbol_exported_and_bound():
    names = _header_functions()
    assert len(names) >= 20
    raw = ctypes.CDLL(q.lib_path())
    for n in names:
        assert hasattr(raw, n), f"{n} declared in include/dsv41q.h but not exported"
    assert set(names) == set(L.PROTOTYPES), set(names) ^ set(L.PROTOTYPES)


def test_host_side_validation_without_gpu():
    lib = L.load()
    # shape errors are reported before any device work
    st = lib.dsv41_dequant_fp8_rows(None, None, 4, 30, 32, None, None)
    assert st == L.BAD_SHAPE and "multiple of block" in L.last_error()
    st = lib.dsv41_gemv_affine(None, 1, 128, None, None, None, 3, 8, 0, None, None, 0, None)
    assert st == L.UNSUPPORTED
    st = lib.dsv41_act_quant_fp8(None, 2, 40, 32, 1, None, None, 0, None, None)
    assert st == L.BAD_SHAPE
    assert lib.dsv41_gemv_workspace_size(32, 4096, 7168) > 32 * 7168 * 2
    assert lib.dsv41_set_wait_limit_ns(10) == L.BAD_ARG          # below 0.1 ms
    assert lib.dsv41_ep_wait(None, 0, None) == L.BAD_ARG
    # the allocation-free GEMV: empty shapes are a no-op (as for the workspace entry point),
    # oversized ones are refused before any device work
    assert lib.dsv41_gemv_fp8_block_noalloc(None, 0, 1024, None, None, 64, L.F32, None, None) == 0
    assert lib.dsv41_gemv_fp8_block_noalloc(None, 4, 1024, None, None, 0, L.F32, None, None) == 0
    assert lib.dsv41_gemv_fp8_block_noalloc(None, 33, 1024, None, None, 64, L.F32, None,
                                            None) == L.UNSUPPORTED
    cfg = L.MoeConfig(dim=7168, inter=2048, n_experts=384, topk=6, score_func=0, gate_temp=1.0,
                      norm_topk_prob=1, route_scale=1.5, swiglu_limit=10.0, flags=1)
    assert lib.dsv41_moe_decode_workspace_size(ctypes.byref(cfg), 64) > 64 * 6 * 7168 * 4


def test_workspaces_stay_proportionate():
    """Scratch is carved only for what the launches use: the split-K fragments of a launch
    that does not split K take no room.  Guards the decode workspace of the BASELINE layer
    (once 11 GB at T=64 and 172 GB at T=4096) and the dense GEMV's (once 3.8 GB at M=4096)."""
    lib = L.load()
    for flags in (1, 1 | L.MOE_PACKED_SCALES):
        cfg = L.MoeConfig(dim=7168, inter=2048, n_experts=384, topk=6, score_func=0,
                          gate_temp=1.0, norm_topk_prob=1, route_scale=1.5, swiglu_limit=10.0,
                          flags=flags)
        for T, cap in ((1, 64e6), (8, 128e6), (64, 512e6), (4096, 4e9)):
            n = lib.dsv41_moe_decode_workspace_size(ctypes.byref(cfg), T)
            assert T * 6 * 7168 * 4 < n < cap, (flags, T, n)
    assert lib.dsv41_gemv_workspace_size(4096, 14336, 7168) < 128e6
    assert lib.dsv41_gemv_workspace_size(1, 4096, 7168) < 16e6
    assert lib.dsv41_moe_route_workspace_size(4096, 7168, 384) <= 4096 * 384 * 4 + 512


def test_errors_map_to_python_exceptions():
    import pytest
    with pytest.raises(ValueError):
        L.check(L.BAD_SHAPE, "x")
    with pytest.raises(q.DSV41Error):
        L.check(L.CUDA_ERR, "x")


def test_no_oracle_import_in_product():
    pkg = os.path.join(ROOT, "deepseek-v41-mlx_b200")
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            src = open(os.path.join(pkg, f)).read()
            assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", src, flags=re.M), f
