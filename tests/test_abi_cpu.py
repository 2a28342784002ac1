"""CPU-only checks of the product boundary: the C-ABI library loads, exports
every symbol include/dw_cuda.h declares, and fails cleanly without a GPU;
host-side quantisation helpers agree with the oracle."""
import ctypes
import os
import re

import numpy as np
import pytest

from dragonwing_edge_rs_b200 import _lib as L
from dragonwing_edge_rs_b200 import quantization as Q
from oracle import dwref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        txt = open(os.path.join(ROOT, "include", h)).read()
        syms |= set(re.findall(r"DW_API\s+[\w\s\*]+?\b(dw_\w+)\s*\(", txt))
    return syms


def test_library_builds_and_loads():
    lib = L.load()
    assert lib.dw_name() == b"cuda-sm100a"


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert len(syms) >= 35
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [s for s in sorted(syms) if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding declares a signature for every one of them
    assert not (syms - set(L.SIGNATURES)), sorted(syms - set(L.SIGNATURES))


def test_no_cuda_fallback_in_product_package():
    """The product package must not import the oracle or run a CPU path."""
    pkg = os.path.join(ROOT, "dragonwing_edge_rs_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                txt = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in txt.replace("oracle/", ""), f


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    out = ctypes.c_void_p()
    st = L.load().dw_create(0, None, ctypes.byref(out))
    assert st in (L.DW_ERR_DEVICE, L.DW_ERR_INVALID_ARG)
    assert not out.value


def test_requant_scales_match_reference_formula():
    rng = np.random.default_rng(1)
    s_w = rng.uniform(0.001, 0.01, 64).astype(np.float32)
    M = Q.requant_scales(0.02, s_w, 0.05)
    for i in range(64):
        assert np.float32(M[i]) == np.float32(dwref.requant_scale(0.02, float(s_w[i]), 0.05))


def test_relu6_ceiling_matches_quantize():
    for s in (0.01, 0.0234, 0.05, 0.047, 0.1):
        assert Q.relu6_ceiling(s) == int(dwref.quantize_f32_to_i8(np.array([6.0], np.float32), s)[0])


def test_roundf_away_matches_oracle():
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.uniform(-130, 130, 20000), np.arange(-130, 130, 0.5),
                        [0.49999997, -0.49999997, 0.5, -0.5]]).astype(np.float32)
    ours = Q.roundf_away(np.clip(x, -128, 127)).astype(np.int32)
    ref = np.array([dwref.lib().dwref_f32_to_i8(float(v)) for v in x], np.int32)
    assert np.array_equal(ours, ref)


def test_per_channel_symmetric_matches_oracle():
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.1, (16, 3, 3, 8)).astype(np.float32)
    q, s = Q.per_channel_symmetric(w)
    s_ref = dwref.per_channel_scales(w.reshape(-1), 16)
    q_ref = dwref.per_channel_quantize(w.reshape(-1), s_ref)
    assert np.array_equal(s, s_ref)
    assert np.array_equal(q.reshape(-1), q_ref)
