"""Loads libqf_moe.so (built in-tree by the package Makefile) and declares the
C ABI of include/qf_moe.h for ctypes.

There is no fallback: if the library is missing or fails to load, every entry
point raises.  The MoE block only runs through the sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libqf_moe.so")

QF_OK = 0
EP_HANDLE_BYTES = 64
STATUS_NAMES = {
    0: "QF_OK", -1: "QF_ERR_ARG", -2: "QF_ERR_CUDA", -3: "QF_ERR_NCCL", -4: "QF_ERR_OOM",
    -5: "QF_ERR_IO", -6: "QF_ERR_TIMEOUT", -7: "QF_ERR_DEVICE", -8: "QF_ERR_UNSUPPORTED",
}


class QfError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class MoEDims(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("experts", C.c_int32), ("top_k", C.c_int32),
                ("intermediate", C.c_int32), ("group", C.c_int32), ("scale_dtype", C.c_int32)]


class MoELayerDesc(C.Structure):
    _fields_ = [("router_w", C.c_void_p), ("router_s", C.c_void_p), ("router_b", C.c_void_p),
                ("coef_w", C.c_void_p), ("coef_s", C.c_void_p), ("coef_b", C.c_void_p),
                ("shared_record", C.c_void_p), ("expert_bank", C.c_void_p),
                ("record_stride", C.c_uint64), ("bank_records", C.c_uint32),
                ("reserved", C.c_uint32)]


class RoutingDesc(C.Structure):
    _fields_ = [("logit_bias", C.c_void_p), ("topk_idx", C.c_void_p), ("topk_w", C.c_void_p),
                ("record_of_pos", C.c_void_p)]


class CacheMetrics(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "capacity", "occupancy", "probationary_occupancy", "protected_occupancy", "hits",
        "misses", "evictions", "fetched_bytes", "prefetch_requests", "useful_prefetch_hits",
        "wasted_prefetches")]


class StoreHeader(C.Structure):
    _fields_ = [("layer_index", C.c_int32), ("experts_per_layer", C.c_int32),
                ("expert_byte_length", C.c_int32), ("payload_byte_length", C.c_uint64),
                ("payload_sha256", C.c_char * 65), ("source_index_sha256", C.c_char * 65)]


class StoreMetrics(C.Structure):
    _fields_ = [("packed_reads", C.c_int64), ("pread_operations", C.c_int64),
                ("read_failures", C.c_int64)]


class LayerHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("router_w", "router_s", "router_b", "coef_w", "coef_s",
                                          "coef_b", "shared_record", "expert_bank")] + \
               [("record_stride", C.c_uint64)]


class StorePackResult(C.Structure):
    _fields_ = [("layers_written", C.c_int32), ("total_bytes", C.c_uint64),
                ("source_index_sha256", C.c_char * 65)]


# (name, restype, argtypes) for every symbol include/qf_moe.h declares.
_P = C.c_void_p
_I = C.c_int32
_S = C.c_int  # qf_status
SIGNATURES = {
    "qf_moe_abi_version": (C.c_int, []),
    "qf_moe_create": (_S, [C.POINTER(MoEDims), C.c_int, C.POINTER(_P)]),
    "qf_moe_destroy": (None, [_P]),
    "qf_moe_set_stream": (_S, [_P, _P]),
    "qf_last_error": (C.c_char_p, [_P]),
    "qf_moe_check": (_S, [_P]),
    "qf_router_logits_q8": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, _P]),
    "qf_router_topk": (_S, [_P, _P, _P, _I, _P, _P]),
    "qf_moe_dispatch_workspace_size": (_S, [_P, _I, C.POINTER(C.c_size_t)]),
    "qf_moe_dispatch_plan": (_S, [_P, _P, _I, _P, _P, _P, _P, C.c_size_t]),
    "qf_moe_workspace_size": (_S, [_P, _I, C.POINTER(C.c_size_t)]),
    "qf_moe_routed_subset": (_S, [_P, C.POINTER(MoELayerDesc), _P, _P, _P, _P, _I, _P, _P, C.c_size_t]),
    "qf_shared_expert": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, _P, _P, C.c_size_t]),
    "qf_moe_combine": (_S, [_P, _I, _P, _P, _P, _P, _P]),
    "qf_moe_grouped_ffn_workspace_size": (_S, [_P, _I, C.POINTER(C.c_size_t)]),
    "qf_moe_grouped_ffn": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, _P, _P, C.c_size_t]),
    "qf_moe_block_forward": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, _P,
                                  C.POINTER(RoutingDesc), _P, _P, _P, C.c_size_t]),
    "qf_moe_stack_forward": (_S, [_P, C.POINTER(MoELayerDesc), _I, _I, _P, _P, _P, C.c_float,
                                  _P, _P, _P, C.c_size_t]),
    "qf_moe_block_forward_static": (_S, [C.c_int32, C.POINTER(MoELayerDesc), _I, _P, _P, _P,
                                         _P, _P, _P]),
    "qf_cache_create": (_S, [_I, _I, C.c_double, _I, C.POINTER(_P)]),
    "qf_cache_destroy": (None, [_P]),
    "qf_cache_acquire": (_S, [_P, _I, _P, _I, _P, _P, C.POINTER(_I), _P, _P, C.POINTER(_I)]),
    "qf_cache_prefetch": (_S, [_P, _I, _P, _I, _P, _P, C.POINTER(_I)]),
    "qf_cache_clear": (_S, [_P]),
    "qf_cache_reset_metrics": (_S, [_P]),
    "qf_cache_get_metrics": (_S, [_P, C.POINTER(CacheMetrics)]),
    "qf_cache_info": (_S, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "qf_cache_layer_slots": (_S, [_P, _P, _P]),
    "qf_cache_layer_metrics": (_S, [_P, _P, _P]),
    "qf_cache_plan_slots": (_S, [_I, C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_uint64)]),
    "qf_tier_create": (_S, [_I, _I, _P, C.c_int64, C.c_uint64, C.POINTER(_P)]),
    "qf_tier_destroy": (None, [_P]),
    "qf_tier_arena": (_S, [_P, C.POINTER(_P), C.POINTER(C.c_uint64)]),
    "qf_tier_fetch": (_S, [_P, _P, _P, _I, _P]),
    "qf_tier_stats": (_S, [_P, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "qf_tier_inject_fault": (_S, [_P, _I, _I]),
    "qf_tier_failed_copies": (_S, [_P, C.POINTER(C.c_int64)]),
    "qf_tier_synchronize": (_S, [_P]),
    "qf_moe_stream_step": (_S, [_P, _P, _P, C.POINTER(MoELayerDesc), _I, _P, _P, _P, _P, _P,
                                C.c_float, _P, C.c_size_t]),
    "qf_ep_create": (_S, [_P, _I, _I, _I, C.POINTER(_P)]),
    "qf_ep_ipc_handle": (_S, [_P, _P]),
    "qf_ep_connect": (_S, [_P, _P]),
    "qf_ep_destroy": (None, [_P]),
    "qf_ep_info": (_S, [_P, C.POINTER(_I), C.POINTER(C.c_int64), C.POINTER(C.c_uint64)]),
    "qf_ep_set_timeout_ms": (_S, [_P, C.c_uint32]),
    "qf_ep_set_down_at_home": (_S, [_P, C.c_int32]),
    "qf_moe_block_forward_ep": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, _P,
                                     C.POINTER(RoutingDesc), _P, _P]),
    "qf_moe_profile_begin": (_S, [_P, _I, _I]),
    "qf_moe_profile_end": (_S, [_P, C.POINTER(C.c_float), C.POINTER(_I)]),
    "qf_synth_records": (_S, [_P, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, _P,
                              C.c_uint64]),
    "qf_synth_router": (_S, [_P, C.c_uint64, C.c_uint32, _P, _P, _P]),
    "qf_synth_coef": (_S, [_P, C.c_uint64, C.c_uint32, _P, _P, _P]),
    "qf_synth_hidden_host": (None, [C.c_uint64, C.c_uint64, _I, _P]),
    "qf_store_header_encode": (_S, [C.POINTER(StoreHeader), _P]),
    "qf_store_header_decode": (_S, [_P, C.c_size_t, C.POINTER(StoreHeader)]),
    "qf_store_validate_manifest": (_S, [C.c_char_p, C.c_size_t]),
    "qf_store_open": (_S, [C.c_char_p, C.c_char_p, C.POINTER(_P)]),
    "qf_store_close": (None, [_P]),
    "qf_store_read_expert": (_S, [_P, _I, _I, _P]),
    "qf_store_load_tier": (_S, [_P, _I, _I, _P, C.c_uint64, _I]),
    "qf_store_get_metrics": (_S, [_P, C.POINTER(StoreMetrics)]),
    "qf_store_verify_layer": (_S, [_P, _I, C.POINTER(_I)]),
    "qf_sha256_hex": (_S, [_P, C.c_size_t, _P]),
    "qf_store_last_error": (C.c_char_p, []),
    "qf_checkpoint_open": (_S, [C.c_char_p, C.POINTER(_P)]),
    "qf_store_pack": (_S, [C.c_char_p, C.c_char_p, _I, C.POINTER(StorePackResult)]),
    "qf_store_verify": (_S, [C.c_char_p, C.c_char_p, C.POINTER(_I)]),
    "qf_lm_head_q4": (_S, [_P, _P, _P, _P, _I, _I, _P, _P]),
    "qf_moe_block_forward_prenorm": (_S, [_P, C.POINTER(MoELayerDesc), _I, _P, _P, C.c_float, _P,
                                          C.POINTER(RoutingDesc), _P, _P, _P, C.c_size_t]),
    "qf_checkpoint_close": (None, [_P]),
    "qf_checkpoint_load_layer": (_S, [_P, _I, C.POINTER(LayerHost), _I, C.POINTER(_I)]),
}

_lib = None


def lib():
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C qwen-fieldfare_b200` "
                "(or __graft_entry__.build()); the MoE path has no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, handle=None) -> None:
    if status != QF_OK:
        msg = lib().qf_last_error(handle).decode() if handle else ""
        raise QfError(status, msg)
