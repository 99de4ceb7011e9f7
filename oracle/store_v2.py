"""Pure-Python restatement of the packed expert store, format v2.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the native
reader (qwen-fieldfare_b200/csrc/qf_store.cu).  The product package never
imports this module.

Restates, from the reference (tanishqpatil/qwen-fieldfare):
  - the layer header: QwenQ4ExpertLayerHeader.encode / .decode
    (Sources/QwenFieldfareCore/Storage/QwenQ4ExpertStore.swift:50-158);
  - the manifest and its validation: QwenQ4ExpertStoreManifest (:24-48) and
    QwenQ4ExpertStore.validateManifest (:322-342);
  - the layer file and its payload digest: QwenQ4ExpertStoreBuilder.packLayer
    (Sources/QwenFieldfareCore/Storage/QwenQ4ExpertStoreBuilder.swift:284-352),
    with the manifest written as pretty-printed JSON with sorted keys (:168-170);
  - the record read: QwenQ4ExpertStore.readExpert (QwenQ4ExpertStore.swift:288-306).
A writer that builds stores of full-size layer files needs no 18 GB: records
that are not given are left as holes of a sparse file (they read as zeros).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct

MAGIC = b"Q4EXP02\x00"
SCHEMA = 2
HEADER_BYTES = 4096
LAYERS = 40
EXPERTS = 256
RECORD_BYTES = 1_769_472
PAYLOAD_BYTES = EXPERTS * RECORD_BYTES
LAYER_FILE_BYTES = HEADER_BYTES + PAYLOAD_BYTES


class StoreError(ValueError):
    pass


def is_sha256(v: str) -> bool:
    """QwenQ4ExpertLayerHeader.isSHA256 (QwenQ4ExpertStore.swift:126-130)."""
    return len(v) == 64 and all(c in "0123456789abcdef" for c in v)


def layer_filename(layer: int) -> str:
    return "layer_%02d.q4exp" % layer


def encode_header(layer_index: int, payload_sha256: str, source_sha256: str,
                  experts: int = EXPERTS, record_bytes: int = RECORD_BYTES,
                  payload_bytes: int = PAYLOAD_BYTES) -> bytes:
    """QwenQ4ExpertStore.swift:76-99."""
    if not (is_sha256(payload_sha256) and is_sha256(source_sha256)):
        raise StoreError("SHA-256 fields must be 64 lowercase hexadecimal characters")
    if not (0 <= layer_index <= 0xFFFFFFFF and 0 < experts <= 0xFFFFFFFF and 0 < record_bytes <= 0xFFFFFFFF):
        raise StoreError("numeric field is out of range")
    b = bytearray(HEADER_BYTES)
    b[0:8] = MAGIC
    struct.pack_into("<IIIII", b, 8, SCHEMA, HEADER_BYTES, layer_index, experts, record_bytes)
    struct.pack_into("<Q", b, 32, payload_bytes)
    b[40:104] = payload_sha256.encode()
    b[104:168] = source_sha256.encode()
    return bytes(b)


def decode_header(b: bytes) -> dict:
    """QwenQ4ExpertStore.swift:101-124."""
    if len(b) != HEADER_BYTES:
        raise StoreError(f"expected {HEADER_BYTES} bytes, got {len(b)}")
    if b[0:8] != MAGIC:
        raise StoreError("magic mismatch")
    schema, hlen, layer, experts, rec = struct.unpack_from("<IIIII", b, 8)
    if schema != SCHEMA:
        raise StoreError("unsupported schema version")
    if hlen != HEADER_BYTES:
        raise StoreError("header byte length mismatch")
    try:
        ph, sh = b[40:104].decode(), b[104:168].decode()
    except UnicodeDecodeError:
        raise StoreError("invalid SHA-256 field")
    if not (is_sha256(ph) and is_sha256(sh)):
        raise StoreError("invalid SHA-256 field")
    return {"layer_index": layer, "experts_per_layer": experts, "expert_byte_length": rec,
            "payload_byte_length": struct.unpack_from("<Q", b, 32)[0],
            "payload_sha256": ph, "source_index_sha256": sh}


def manifest(source_sha256: str, payload_hashes: list[str]) -> dict:
    return {"schemaVersion": SCHEMA, "sourceIndexSHA256": source_sha256,
            "layers": [{"layerIndex": i, "filename": layer_filename(i), "fileSize": LAYER_FILE_BYTES,
                        "payloadSHA256": h} for i, h in enumerate(payload_hashes)]}


def manifest_text(m: dict) -> str:
    """Pretty-printed with sorted keys, as the builder writes it (QwenQ4ExpertStoreBuilder.swift:168-170)."""
    return json.dumps(m, indent=2, sort_keys=True)


def validate_manifest(m: dict) -> None:
    """QwenQ4ExpertStore.swift:322-342."""
    if m.get("schemaVersion") != SCHEMA:
        raise StoreError(f"unsupported schema version {m.get('schemaVersion')}")
    if not is_sha256(m.get("sourceIndexSHA256", "")):
        raise StoreError("invalid source index SHA-256")
    layers = m.get("layers", [])
    if len(layers) != LAYERS:
        raise StoreError(f"expected {LAYERS} layers, got {len(layers)}")
    for expected, layer in enumerate(sorted(layers, key=lambda e: e["layerIndex"])):
        if (layer["layerIndex"] != expected or layer["filename"] != layer_filename(expected)
                or layer["fileSize"] != LAYER_FILE_BYTES or not is_sha256(layer["payloadSHA256"])):
            raise StoreError(f"invalid layer entry {expected}")


def payload_sha256(records: dict[int, bytes]) -> str:
    """SHA-256 of the 256 records in expert order; absent records are zeros."""
    h = hashlib.sha256()
    zero = bytes(RECORD_BYTES)
    for e in range(EXPERTS):
        h.update(records.get(e, zero))
    return h.hexdigest()


def write_store(directory: str, source_sha256: str, records: dict[tuple[int, int], bytes],
                hash_layers: tuple[int, ...] = ()) -> list[str]:
    """Writes manifest.json and the 40 full-size (sparse) layer files.

    records maps (layer, expert) -> 1,769,472 bytes.  The payload digest is
    computed for the layers in hash_layers (hashing a layer reads 453 MB);
    the others get a placeholder digest of their layer number, which the
    reader does not check unless asked to verify that layer."""
    os.makedirs(directory, exist_ok=True)
    hashes = []
    for layer in range(LAYERS):
        mine = {e: r for (l, e), r in records.items() if l == layer}
        digest = payload_sha256(mine) if layer in hash_layers else ("%064x" % (layer + 1))
        hashes.append(digest)
        path = os.path.join(directory, layer_filename(layer))
        with open(path, "wb") as f:
            f.truncate(LAYER_FILE_BYTES)
            f.write(encode_header(layer, digest, source_sha256))
            for e, rec in mine.items():
                assert len(rec) == RECORD_BYTES
                f.seek(HEADER_BYTES + e * RECORD_BYTES)
                f.write(rec)
    with open(os.path.join(directory, "manifest.json"), "w") as f:
        f.write(manifest_text(manifest(source_sha256, hashes)))
    return hashes


def read_expert(directory: str, layer: int, expert: int) -> bytes:
    with open(os.path.join(directory, layer_filename(layer)), "rb") as f:
        f.seek(HEADER_BYTES + expert * RECORD_BYTES)
        return f.read(RECORD_BYTES)
