"""Packed expert store (format v2): the native reader (qf_store_*) against the
reference's own store tests and the Python restatement oracle/store_v2.py.

The first three tests port Tests/QwenFieldfareCore/Storage/QwenQ4ExpertStoreTests.swift
(:11-24 header round trip, :26-49 corrupt magic and invalid digest, :51-85
manifest with every layer exactly once).  The store I/O tests build full-size
layer files as sparse files, so the 18 GB geometry costs a few MB of disk.
No GPU is used."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import store_v2 as O  # noqa: E402

from qfmoe import QfError  # noqa: E402
from qfmoe import store as S  # noqa: E402

PAYLOAD = "a" * 64
SOURCE = "b" * 64


# ---- ports of the reference's store tests ---------------------------------

def test_layer_header_round_trips_without_native_alignment_assumptions():
    enc = S.encode_header(17, PAYLOAD, SOURCE)
    assert len(enc) == S.HEADER_BYTES
    dec = S.decode_header(enc)
    assert dec == {"layer_index": 17, "experts_per_layer": 256, "expert_byte_length": 1_769_472,
                   "payload_byte_length": 256 * 1_769_472, "payload_sha256": PAYLOAD,
                   "source_index_sha256": SOURCE}
    # byte-identical to the restated encoder
    assert enc == O.encode_header(17, PAYLOAD, SOURCE)


def test_layer_header_rejects_corrupt_magic_and_digest():
    enc = bytearray(S.encode_header(0, PAYLOAD, SOURCE))
    enc[0] ^= 0xFF
    with pytest.raises(QfError, match="magic"):
        S.decode_header(bytes(enc))
    with pytest.raises(QfError, match="SHA-256"):
        S.encode_header(0, "z" * 64, SOURCE)


def test_manifest_requires_every_canonical_layer_exactly_once():
    valid = O.manifest(SOURCE, [PAYLOAD] * 40)
    S.validate_manifest(O.manifest_text(valid))
    missing = dict(valid, layers=valid["layers"][:-1])
    with pytest.raises(QfError):
        S.validate_manifest(json.dumps(missing))
    dup_layers = list(valid["layers"])
    dup_layers[39] = dup_layers[38]
    with pytest.raises(QfError):
        S.validate_manifest(json.dumps(dict(valid, layers=dup_layers)))
    for m in (missing, dict(valid, layers=dup_layers)):
        with pytest.raises(O.StoreError):
            O.validate_manifest(m)


# ---- header and manifest edge cases, native vs restatement -----------------

@pytest.mark.parametrize("mutate", ["short", "schema", "hlen", "hexcase", "hexchar"])
def test_header_decode_rejects_what_the_reference_rejects(mutate):
    b = bytearray(O.encode_header(3, PAYLOAD, SOURCE))
    if mutate == "short":
        b = b[:-1]
    elif mutate == "schema":
        b[8] = 3
    elif mutate == "hlen":
        b[13] = 0
    elif mutate == "hexcase":
        b[40] = ord("A")
    elif mutate == "hexchar":
        b[110] = ord("g")
    with pytest.raises(QfError):
        S.decode_header(bytes(b))
    with pytest.raises(O.StoreError):
        O.decode_header(bytes(b))


def test_header_fields_are_little_endian_at_the_reference_offsets():
    b = S.encode_header(0x01020304, PAYLOAD, SOURCE, experts_per_layer=0x0A0B0C0D,
                        expert_byte_length=0x11223344, payload_byte_length=0x0102030405060708)
    assert b[:8] == b"Q4EXP02\x00"
    assert b[8:16] == bytes([2, 0, 0, 0, 0, 16, 0, 0])
    assert b[16:20] == bytes([4, 3, 2, 1]) and b[20:24] == bytes([0x0D, 0x0C, 0x0B, 0x0A])
    assert b[24:28] == bytes([0x44, 0x33, 0x22, 0x11]) and b[28:32] == bytes(4)
    assert b[32:40] == bytes([8, 7, 6, 5, 4, 3, 2, 1])
    assert b[168:] == bytes(4096 - 168)


def test_manifest_edge_cases():
    base = O.manifest(SOURCE, ["%064x" % i for i in range(40)])
    # any key order, compact or pretty, layers in any order
    shuffled = dict(base, layers=list(reversed(base["layers"])))
    S.validate_manifest(json.dumps(shuffled, separators=(",", ":")))
    bad = [dict(base, schemaVersion=1), dict(base, sourceIndexSHA256="B" * 64)]
    for field, value in (("filename", "layer_5.q4exp"), ("fileSize", O.LAYER_FILE_BYTES - 1),
                         ("payloadSHA256", "0" * 63)):
        layers = [dict(e) for e in base["layers"]]
        layers[5][field] = value
        bad.append(dict(base, layers=layers))
    for m in bad:
        with pytest.raises(QfError):
            S.validate_manifest(json.dumps(m))
        with pytest.raises(O.StoreError):
            O.validate_manifest(m)
    for text in ("", "[]", "{", '{"schemaVersion": "2"}', json.dumps(base) + "x"):
        with pytest.raises(QfError):
            S.validate_manifest(text)


def test_sha256_known_answers_and_block_boundaries():
    # FIPS 180-4 examples (one block, empty, two blocks)
    assert S.sha256_hex(b"abc") == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert S.sha256_hex(b"") == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    assert S.sha256_hex(b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq") == \
        "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"
    rng = np.random.default_rng(5)
    for n in (1, 55, 56, 63, 64, 65, 119, 120, 4095, 1 << 20):
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert S.sha256_hex(d) == hashlib.sha256(d).hexdigest(), n


# ---- store I/O on sparse full-size layer files -----------------------------

def _records(seed, keys):
    rng = np.random.default_rng(seed)
    return {k: rng.integers(0, 256, O.RECORD_BYTES, dtype=np.uint8).tobytes() for k in keys}


@pytest.fixture(scope="module")
def store(tmp_path_factory):
    root = tmp_path_factory.mktemp("model")
    index = root / "model.safetensors.index.json"
    index.write_text('{"weight_map": {}}\n')
    src = hashlib.sha256(index.read_bytes()).hexdigest()
    recs = _records(11, [(0, 0), (0, 255), (1, 7), (1, 200), (39, 3), (39, 128)])
    d = root / "qwen_q4_experts"
    O.write_store(str(d), src, recs, hash_layers=(1,))
    return str(d), str(index), recs


def test_open_read_and_metrics(store):
    d, index, recs = store
    with S.ExpertStore(d, index) as s:
        for (layer, expert), rec in recs.items():
            got = s.read_expert(layer, expert)
            assert got.tobytes() == rec == O.read_expert(d, layer, expert)
        assert not s.read_expert(0, 1).any()  # a hole reads as zeros
        for bad in ((40, 0), (-1, 0), (0, 256), (5, -1)):
            with pytest.raises(QfError, match="QF_ERR_ARG"):
                s.read_expert(*bad)
        m = s.metrics()
    assert m == {"kind": "qwen-q4-packed-v2", "packed_reads": len(recs) + 1,
                 "packed_pread_operations": len(recs) + 1, "packed_read_failures": 4}


def test_open_without_source_check(store):
    d, _, recs = store
    with S.ExpertStore(d) as s:
        assert s.read_expert(39, 3).tobytes() == recs[(39, 3)]


def test_open_rejects_a_different_source_index(store, tmp_path):
    d, _, _ = store
    other = tmp_path / "model.safetensors.index.json"
    other.write_text('{"weight_map": {"x": "y"}}\n')
    with pytest.raises(QfError, match="source mismatch"):
        S.ExpertStore(d, str(other))


def test_verify_layer_checks_the_payload_digest(store):
    d, index, _ = store
    with S.ExpertStore(d, index) as s:
        assert s.verify_layer(1)        # digest written from the records
        assert not s.verify_layer(0)    # placeholder digest


def test_load_tier_fills_records_in_layer_major_order(store):
    d, index, recs = store
    tier = np.zeros((256, O.RECORD_BYTES + 64), dtype=np.uint8)  # stride above one record
    tier[:, O.RECORD_BYTES:] = 0xAB
    with S.ExpertStore(d, index) as s:
        s.load_tier(tier, first_layer=39, n_layers=1, threads=4)
        m = s.metrics()
    assert tier[3, :O.RECORD_BYTES].tobytes() == recs[(39, 3)]
    assert tier[128, :O.RECORD_BYTES].tobytes() == recs[(39, 128)]
    assert not tier[0, :O.RECORD_BYTES].any() and not tier[255, :O.RECORD_BYTES].any()
    assert (tier[:, O.RECORD_BYTES:] == 0xAB).all()  # padding past each record untouched
    assert m["packed_reads"] == 256 and m["packed_read_failures"] == 0
    with S.ExpertStore(d) as s:
        with pytest.raises(ValueError):
            s.load_tier(tier, first_layer=38, n_layers=2)  # tier too small for two layers
        with pytest.raises(QfError):
            s.load_tier(tier[:, :O.RECORD_BYTES + 64], first_layer=40, n_layers=1)


def _copy_store(src, dst):
    os.makedirs(dst)
    for name in os.listdir(src):
        if name.endswith(".q4exp"):
            # header only: the copy keeps the size as a hole
            with open(os.path.join(src, name), "rb") as f:
                head = f.read(O.HEADER_BYTES)
            with open(os.path.join(dst, name), "wb") as f:
                f.truncate(O.LAYER_FILE_BYTES)
                f.write(head)
        else:
            with open(os.path.join(src, name), "rb") as f, open(os.path.join(dst, name), "wb") as g:
                g.write(f.read())


@pytest.mark.parametrize("damage", ["truncate", "header_layer", "header_digest", "no_manifest", "missing_file"])
def test_open_rejects_damaged_stores(store, tmp_path, damage):
    d, _, _ = store
    c = str(tmp_path / "copy")
    _copy_store(d, c)
    f7 = os.path.join(c, O.layer_filename(7))
    if damage == "truncate":
        os.truncate(f7, O.LAYER_FILE_BYTES - 1)
    elif damage in ("header_layer", "header_digest"):
        m = json.load(open(os.path.join(c, "manifest.json")))
        src = m["sourceIndexSHA256"]
        digest = m["layers"][7]["payloadSHA256"]
        hdr = O.encode_header(8, digest, src) if damage == "header_layer" else \
            O.encode_header(7, "c" * 64, src)
        with open(f7, "r+b") as f:
            f.write(hdr)
    elif damage == "no_manifest":
        os.remove(os.path.join(c, "manifest.json"))
    else:
        os.remove(f7)
    with pytest.raises(QfError):
        S.ExpertStore(c)


def test_sha256_portable_rounds_match_the_accelerated_ones():
    """The library hashes with the x86 SHA extensions where the CPU has them;
    QF_SHA256_PORTABLE=1 selects the FIPS 180-4 rounds.  Both give hashlib's
    digests (run in a child process: the choice is made once per process)."""
    import subprocess
    code = ("import hashlib, numpy as np; from qfmoe import store as S; "
            "rng = np.random.default_rng(3); "
            "ok = all(S.sha256_hex(d) == hashlib.sha256(d).hexdigest() for d in "
            "[rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in (0, 3, 64, 65, 1000, 1 << 18)]); "
            "print('ok' if ok else 'bad')")
    env = dict(os.environ, QF_SHA256_PORTABLE="1",
               PYTHONPATH=os.path.join(ROOT, "qwen-fieldfare_b200") + os.pathsep + os.environ.get("PYTHONPATH", ""))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert out.stdout.strip() == "ok", out.stderr
