"""The C ABI library loads without a GPU and exports every entry point that
include/qf_moe.h declares, and the ctypes table in qfmoe._lib covers them all.
No compute call is made here (no GPU in the CPU suite)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qf_moe.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for must in ("qf_moe_create", "qf_moe_block_forward", "qf_moe_stack_forward",
                 "qf_router_logits_q8", "qf_router_topk", "qf_moe_dispatch_plan"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    from qfmoe._lib import LIB_PATH, SIGNATURES, lib
    L = lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(SIGNATURES) == declared_symbols()
    assert L.qf_moe_abi_version() == 1
    assert os.path.dirname(LIB_PATH).endswith("qfmoe")


def test_create_without_gpu_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from qfmoe._lib import MoEDims, lib
    dims = MoEDims(2048, 256, 8, 512, 64, 0)
    h = C.c_void_p()
    assert lib().qf_moe_create(C.byref(dims), 0, C.byref(h)) != 0
    assert not h.value
    bad = MoEDims(4096, 256, 8, 512, 64, 0)
    assert lib().qf_moe_create(C.byref(bad), 0, C.byref(h)) == -1  # QF_ERR_ARG
