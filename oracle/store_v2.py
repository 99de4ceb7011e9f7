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
  - the MLX checkpoint the reference runs: safetensors shards behind
    model.safetensors.index.json, tensor names and shapes of one MoE layer
    (Sources/QwenFieldfareCore/Runtime/Generation/QwenQ4ActiveExpertStreamingRunner.swift:596-620;
    switch_mlp slices per expert, QwenQ4ExpertStoreBuilder.swift:41-55, 202-282).
Writers that build full-size files need no 18 GB: records and slices that are
not given are left as holes of a sparse file (they read as zeros).
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


# ---- MLX safetensors checkpoint -------------------------------------------

# record components: (suffix, bytes, MLX shape of one expert's tensor, is 16-bit)
COMPONENTS = [
    ("gate_proj.weight", 524_288, (512, 256), False), ("gate_proj.scales", 32_768, (512, 32), True),
    ("gate_proj.biases", 32_768, (512, 32), True),
    ("up_proj.weight", 524_288, (512, 256), False), ("up_proj.scales", 32_768, (512, 32), True),
    ("up_proj.biases", 32_768, (512, 32), True),
    ("down_proj.weight", 524_288, (2048, 64), False), ("down_proj.scales", 32_768, (2048, 8), True),
    ("down_proj.biases", 32_768, (2048, 8), True),
]
COMPONENT_OFFSETS = [0, 524_288, 557_056, 589_824, 1_114_112, 1_146_880, 1_179_648, 1_703_936, 1_736_704]


class Sparse:
    """A tensor of `size` bytes of which only `pieces` {offset: bytes} are data."""

    def __init__(self, size: int, pieces: dict[int, bytes]):
        self.size, self.pieces = size, pieces


def split_record(record: bytes) -> list[bytes]:
    return [record[o:o + n] for o, (_, n, _, _) in zip(COMPONENT_OFFSETS, COMPONENTS)]


def moe_layer_tensors(layer: int, router_w: bytes, router_s: bytes, router_b: bytes, coef_w: bytes,
                      coef_s: bytes, coef_b: bytes, shared_record: bytes, bank: dict[int, bytes],
                      scale_dtype: str = "F16") -> dict:
    """name -> (dtype, shape, bytes | Sparse) for one layer's MoE tensors."""
    pre = f"language_model.model.layers.{layer}.mlp."
    t = {pre + "gate.weight": ("U32", (256, 512), router_w),
         pre + "gate.scales": (scale_dtype, (256, 32), router_s),
         pre + "gate.biases": (scale_dtype, (256, 32), router_b),
         pre + "shared_expert_gate.weight": ("U32", (1, 512), coef_w),
         pre + "shared_expert_gate.scales": (scale_dtype, (1, 32), coef_s),
         pre + "shared_expert_gate.biases": (scale_dtype, (1, 32), coef_b)}
    for (suffix, n, shape, is16), part in zip(COMPONENTS, split_record(shared_record)):
        t[pre + "shared_expert." + suffix] = (scale_dtype if is16 else "U32", shape, part)
    for k, (suffix, n, shape, is16) in enumerate(COMPONENTS):
        pieces = {e * n: split_record(rec)[k] for e, rec in bank.items()}
        t[pre + "switch_mlp." + suffix] = (scale_dtype if is16 else "U32", (256,) + shape,
                                           Sparse(256 * n, pieces))
    return t


def write_safetensors(path: str, tensors: dict) -> None:
    """safetensors: u64 little-endian header length, JSON header with
    data_offsets relative to the data, header padded with spaces to 8 bytes."""
    header, off = {}, 0
    for name, (dtype, shape, data) in tensors.items():
        n = data.size if isinstance(data, Sparse) else len(data)
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * (-len(hj) % 8)
    base = 8 + len(hj)
    with open(path, "wb") as f:
        f.truncate(base + off)
        f.write(struct.pack("<Q", len(hj)) + hj)
        for name, (dtype, shape, data) in tensors.items():
            start = base + header[name]["data_offsets"][0]
            if isinstance(data, Sparse):
                for o, piece in data.pieces.items():
                    f.seek(start + o)
                    f.write(piece)
            else:
                f.seek(start)
                f.write(data)


def write_checkpoint(model_dir: str, tensors: dict, n_shards: int = 2) -> None:
    """Tensors spread round-robin over n_shards files, with the index."""
    os.makedirs(model_dir, exist_ok=True)
    names = list(tensors)
    shard_names = [f"model-{i + 1:05d}-of-{n_shards:05d}.safetensors" for i in range(n_shards)]
    weight_map = {}
    for i, sn in enumerate(shard_names):
        mine = {n: tensors[n] for n in names[i::n_shards]}
        write_safetensors(os.path.join(model_dir, sn), mine)
        weight_map.update({n: sn for n in mine})
    with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f, indent=2)
