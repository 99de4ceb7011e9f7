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


def _good_desc():
    """A descriptor with fake but well-aligned addresses (never dereferenced:
    every check below fails before any CUDA call)."""
    from qfmoe._lib import MoELayerDesc
    base = 1 << 40
    return MoELayerDesc(base, base + 0x100000, base + 0x200000, base + 0x300000,
                        base + 0x400000, base + 0x500000, base + 0x600000, base + 0x1000000,
                        1769472, 256, 0)


BAD_DESCRIPTORS = [
    ("coef_w + 8", lambda d: setattr(d, "coef_w", d.coef_w + 8)),
    ("router_w + 4", lambda d: setattr(d, "router_w", d.router_w + 4)),
    ("router_s + 2", lambda d: setattr(d, "router_s", d.router_s + 2)),
    ("coef_s + 1", lambda d: setattr(d, "coef_s", d.coef_s + 1)),
    ("coef_b + 1", lambda d: setattr(d, "coef_b", d.coef_b + 1)),
    ("shared_record + 16", lambda d: setattr(d, "shared_record", d.shared_record + 16)),
    ("expert_bank + 16", lambda d: setattr(d, "expert_bank", d.expert_bank + 16)),
    ("record_stride 1769472 + 16", lambda d: setattr(d, "record_stride", 1769472 + 16)),
    ("record_stride too small", lambda d: setattr(d, "record_stride", 1769472 - 32)),
    ("bank_records 0", lambda d: setattr(d, "bank_records", 0)),
    ("bank_records 2^23", lambda d: setattr(d, "bank_records", 1 << 23)),
    ("reserved", lambda d: setattr(d, "reserved", 1)),
    ("coef_b NULL", lambda d: setattr(d, "coef_b", None)),
]


@pytest.mark.parametrize("name,spoil", BAD_DESCRIPTORS, ids=[b[0] for b in BAD_DESCRIPTORS])
def test_static_entry_rejects_bad_descriptors_before_any_cuda_call(name, spoil):
    """qf_moe_block_forward_static applies qf_moe_block_forward's descriptor
    rules (16-byte router/coefficient codes, 32-byte records, stride a multiple
    of 32, ...) and returns QF_ERR_ARG without touching the device: on this
    GPU-less machine a good descriptor reaches cudaGetDevice and gets
    QF_ERR_CUDA instead."""
    from qfmoe._lib import lib
    x = 1 << 41
    out = (1 << 41) + (1 << 20)
    d = _good_desc()
    spoil(d)
    assert lib().qf_moe_block_forward_static(0, C.byref(d), 1, x, None, out, None, None,
                                             None) == -1, name


def test_static_entry_good_descriptor_passes_the_checks():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from qfmoe._lib import lib
    d = _good_desc()
    x = 1 << 41
    out = (1 << 41) + (1 << 20)
    assert lib().qf_moe_block_forward_static(0, C.byref(d), 1, x, None, out, None, None,
                                             None) == -2  # QF_ERR_CUDA: no device here
    assert lib().qf_moe_block_forward_static(0, C.byref(d), 1, x + 8, None, out, None, None,
                                             None) == -1  # x must be 16-byte aligned
