"""Packed expert store (format v2): the reference's per-layer expert files as
the source of the pinned-host tier (include/qf_moe.h, qf_store_*).

The store directory holds manifest.json and layer_00.q4exp .. layer_39.q4exp;
each layer file is a 4,096-byte header and 256 records of 1,769,472 bytes in
expert order -- the HBM slot layout, so records go to the tier unchanged
(Sources/QwenFieldfareCore/Storage/QwenQ4ExpertStore.swift:50-316).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._lib import QF_OK, LayerHost, QfError, StoreHeader, StoreMetrics, lib
from .moe import EXPERTS, RECORD_BYTES

HEADER_BYTES = 4096
LAYERS = 40
PAYLOAD_BYTES = EXPERTS * RECORD_BYTES
LAYER_FILE_BYTES = HEADER_BYTES + PAYLOAD_BYTES


def _ok(status: int) -> None:
    if status != QF_OK:
        raise QfError(status, lib().qf_store_last_error().decode())


def layer_filename(layer: int) -> str:
    """QwenQ4ExpertStore.layerFilename (QwenQ4ExpertStore.swift:200-202)."""
    return f"layer_{layer:02d}.q4exp"


def sha256_hex(data) -> str:
    """SHA-256 (FIPS 180-4) of a bytes-like object, by the library."""
    buf = np.frombuffer(memoryview(data), dtype=np.uint8)
    out = C.create_string_buffer(65)
    _ok(lib().qf_sha256_hex(C.c_void_p(buf.ctypes.data), buf.size, out))
    return out.value.decode()


def encode_header(layer_index: int, payload_sha256: str, source_index_sha256: str,
                  experts_per_layer: int = EXPERTS, expert_byte_length: int = RECORD_BYTES,
                  payload_byte_length: int = PAYLOAD_BYTES) -> bytes:
    """QwenQ4ExpertLayerHeader.encode (QwenQ4ExpertStore.swift:76-99)."""
    h = StoreHeader(layer_index, experts_per_layer, expert_byte_length, payload_byte_length,
                    payload_sha256.encode(), source_index_sha256.encode())
    out = (C.c_uint8 * HEADER_BYTES)()
    _ok(lib().qf_store_header_encode(C.byref(h), out))
    return bytes(out)


def decode_header(data: bytes) -> dict:
    """QwenQ4ExpertLayerHeader.decode (QwenQ4ExpertStore.swift:101-124)."""
    buf = (C.c_uint8 * len(data)).from_buffer_copy(data)
    h = StoreHeader()
    _ok(lib().qf_store_header_decode(buf, len(data), C.byref(h)))
    return {"layer_index": h.layer_index, "experts_per_layer": h.experts_per_layer,
            "expert_byte_length": h.expert_byte_length,
            "payload_byte_length": h.payload_byte_length,
            "payload_sha256": h.payload_sha256.decode(),
            "source_index_sha256": h.source_index_sha256.decode()}


def validate_manifest(text: str | bytes) -> None:
    """QwenQ4ExpertStore.validateManifest (QwenQ4ExpertStore.swift:322-342)."""
    raw = text.encode() if isinstance(text, str) else bytes(text)
    _ok(lib().qf_store_validate_manifest(raw, len(raw)))


class ExpertStore:
    """An opened store (QwenQ4ExpertStore.init, QwenQ4ExpertStore.swift:213-282).

    source_index: path of the checkpoint's model.safetensors.index.json, whose
    SHA-256 must match the manifest; None skips that check."""

    def __init__(self, directory: str, source_index: str | None = None):
        h = C.c_void_p()
        _ok(lib().qf_store_open(os.fsencode(directory),
                                os.fsencode(source_index) if source_index else None, C.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            lib().qf_store_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def read_expert(self, layer: int, expert: int, out: np.ndarray | None = None) -> np.ndarray:
        """One record as uint8 [1,769,472] (readExpert, QwenQ4ExpertStore.swift:288-306)."""
        if out is None:
            out = np.empty(RECORD_BYTES, dtype=np.uint8)
        if out.dtype != np.uint8 or out.nbytes < RECORD_BYTES or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous uint8 array of >= 1769472 bytes")
        _ok(lib().qf_store_read_expert(self.h, layer, expert, C.c_void_p(out.ctypes.data)))
        return out

    def load_tier(self, host_records, first_layer: int = 0, n_layers: int = LAYERS,
                  threads: int = 8) -> None:
        """Fill a host tier (uint8 [n_layers * 256, >= RECORD_BYTES], numpy array or
        CPU torch tensor, pinned for asynchronous copies): record index
        (layer - first_layer) * 256 + expert."""
        if hasattr(host_records, "data_ptr"):
            ptr, shape, stride = host_records.data_ptr(), tuple(host_records.shape), host_records.stride(0)
            ok = host_records.dtype.__str__() == "torch.uint8" and host_records.stride(1) == 1
        else:
            ptr, shape, stride = host_records.ctypes.data, host_records.shape, host_records.strides[0]
            ok = host_records.dtype == np.uint8 and host_records.strides[1] == 1
        if not ok or len(shape) != 2 or shape[1] < RECORD_BYTES or shape[0] < n_layers * EXPERTS:
            raise ValueError("host_records must be uint8 [>= n_layers * 256, >= 1769472], rows contiguous")
        _ok(lib().qf_store_load_tier(self.h, first_layer, n_layers, C.c_void_p(ptr), stride, threads))

    def verify_layer(self, layer: int) -> bool:
        """Payload SHA-256 of one layer against the manifest."""
        m = C.c_int32()
        _ok(lib().qf_store_verify_layer(self.h, layer, C.byref(m)))
        return bool(m.value)

    def metrics(self) -> dict:
        """metricsSnapshot (QwenQ4ExpertStore.swift:308-316)."""
        m = StoreMetrics()
        _ok(lib().qf_store_get_metrics(self.h, C.byref(m)))
        return {"kind": "qwen-q4-packed-v2", "packed_reads": m.packed_reads,
                "packed_pread_operations": m.pread_operations,
                "packed_read_failures": m.read_failures}


class Checkpoint:
    """The MoE tensors of an MLX safetensors checkpoint (qf_checkpoint_*): the
    directory holds model.safetensors.index.json and its shards
    (QwenQ4ActiveExpertStreamingRunner.swift:596-620)."""

    def __init__(self, model_path: str):
        h = C.c_void_p()
        _ok(lib().qf_checkpoint_open(os.fsencode(model_path), C.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            lib().qf_checkpoint_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_layer(self, layer: int, with_bank: bool = True, threads: int = 8):
        """One layer in the host layout of qf_moe_layer: a dict of uint8 numpy
        arrays (router_w, router_s, router_b, coef_w, coef_s, coef_b, shared,
        bank [256, RECORD_BYTES] or None) and the scale dtype ("bf16" | "f16")."""
        out = {"router_w": np.empty(EXPERTS * 2048, np.uint8),
               "router_s": np.empty(EXPERTS * 64, np.uint8), "router_b": np.empty(EXPERTS * 64, np.uint8),
               "coef_w": np.empty(2048, np.uint8), "coef_s": np.empty(64, np.uint8),
               "coef_b": np.empty(64, np.uint8), "shared": np.empty(RECORD_BYTES, np.uint8),
               "bank": np.empty((EXPERTS, RECORD_BYTES), np.uint8) if with_bank else None}
        ptr = {k: (C.c_void_p(v.ctypes.data) if v is not None else None) for k, v in out.items()}
        d = LayerHost(ptr["router_w"], ptr["router_s"], ptr["router_b"], ptr["coef_w"], ptr["coef_s"],
                      ptr["coef_b"], ptr["shared"], ptr["bank"], RECORD_BYTES)
        dt = C.c_int32()
        _ok(lib().qf_checkpoint_load_layer(self.h, layer, C.byref(d), threads, C.byref(dt)))
        return out, ("bf16" if dt.value == 1 else "f16")

    def layer_weights(self, ctx, layer: int, threads: int = 8):
        """The layer as device-resident MoELayerWeights, and its scale dtype."""
        import torch
        from .moe import MoELayerWeights
        host, dtype = self.load_layer(layer, True, threads)
        if (dtype == "bf16") != bool(ctx.scale_bf16):
            raise ValueError(f"checkpoint scales are {dtype}; create the MoEContext with "
                             f"scale_bf16={dtype == 'bf16'}")
        dev = ctx.device

        def up(a, i16=False):
            t = torch.from_numpy(a)
            return (t.view(torch.int16) if i16 else t).to(dev)
        return MoELayerWeights(up(host["router_w"]), up(host["router_s"], True), up(host["router_b"], True),
                               up(host["coef_w"]), up(host["coef_s"], True), up(host["coef_b"], True),
                               up(host["shared"]), up(host["bank"])), dtype


def pack_store(model_path: str, out_dir: str | None = None, resume: bool = False) -> dict:
    """Build the v2 store from the checkpoint's switch_mlp tensors
    (QwenQ4ExpertStoreBuilder.pack; qf_store_pack)."""
    from ._lib import StorePackResult
    r = StorePackResult()
    _ok(lib().qf_store_pack(os.fsencode(model_path), os.fsencode(out_dir) if out_dir else None, int(resume),
                            C.byref(r)))
    return {"layers_written": r.layers_written, "total_bytes": r.total_bytes,
            "source_index_sha256": r.source_index_sha256.decode()}


def verify_store(model_path: str, out_dir: str | None = None) -> int:
    """Every layer's header and payload SHA-256 (QwenQ4ExpertStoreBuilder.verify)."""
    n = C.c_int32()
    _ok(lib().qf_store_verify(os.fsencode(model_path), os.fsencode(out_dir) if out_dir else None, C.byref(n)))
    return n.value
