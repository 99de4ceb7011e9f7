"""Store builder (qf_store_pack / qf_store_verify): a 40-layer checkpoint of
switch_mlp tensors (sparse safetensors shards written by oracle/store_v2.py)
packed into the v2 store at full geometry, read back against the records the
shards hold, its manifest and digests checked against the restatement, then
the builder's second call, verification, resume after an interrupted pack and
a changed source index.  No GPU is used; the layer files stay sparse."""
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

DATA = {(0, 0), (0, 255), (7, 3), (39, 100)}


def _checkpoint(d):
    rng = np.random.default_rng(44)
    recs = {k: rng.integers(0, 256, O.RECORD_BYTES, dtype=np.uint8).tobytes() for k in sorted(DATA)}
    tensors = {}
    for layer in range(40):
        pre = f"language_model.model.layers.{layer}.mlp.switch_mlp."
        for k, (suffix, n, shape, is16) in enumerate(O.COMPONENTS):
            pieces = {e * n: O.split_record(r)[k] for (l, e), r in recs.items() if l == layer}
            tensors[pre + suffix] = ("F16" if is16 else "U32", (256,) + shape, O.Sparse(256 * n, pieces))
    O.write_checkpoint(d, tensors, n_shards=4)
    return recs


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("mlx_ckpt"))
    recs = _checkpoint(d)
    r = S.pack_store(d)
    return d, recs, r


def test_pack_builds_the_store_the_reader_opens(packed):
    d, recs, r = packed
    index = os.path.join(d, "model.safetensors.index.json")
    src = hashlib.sha256(open(index, "rb").read()).hexdigest()
    assert r == {"layers_written": 40, "total_bytes": 40 * O.LAYER_FILE_BYTES, "source_index_sha256": src}
    out = os.path.join(d, "qwen_q4_experts")
    assert sorted(os.listdir(out)) == sorted(["manifest.json"] + [O.layer_filename(i) for i in range(40)])
    m = json.load(open(os.path.join(out, "manifest.json")))
    O.validate_manifest(m)
    assert m["sourceIndexSHA256"] == src
    digests = {e["layerIndex"]: e["payloadSHA256"] for e in m["layers"]}
    assert digests[7] == O.payload_sha256({3: recs[(7, 3)]})
    assert digests[12] == O.payload_sha256({})
    with S.ExpertStore(out, index) as s:
        for (l, e), rec in recs.items():
            assert s.read_expert(l, e).tobytes() == rec
        assert not s.read_expert(7, 4).any()
        assert s.verify_layer(0) and s.verify_layer(39)
    for l in range(40):
        hdr = O.decode_header(open(os.path.join(out, O.layer_filename(l)), "rb").read(O.HEADER_BYTES))
        assert hdr["layer_index"] == l and hdr["payload_sha256"] == digests[l] and hdr["source_index_sha256"] == src


def test_second_pack_opens_the_existing_store_and_verify_checks_every_layer(packed):
    d, _, _ = packed
    assert S.pack_store(d)["layers_written"] == 0
    assert S.verify_store(d) == 40


def test_resume_after_an_interrupted_pack(packed, tmp_path):
    d, recs, _ = packed
    out = str(tmp_path / "store")
    src_out = os.path.join(d, "qwen_q4_experts")
    m = json.load(open(os.path.join(src_out, "manifest.json")))
    os.makedirs(out)
    # layers 0..4 completed and checkpointed, layer 5 half written
    for l in range(5):
        os.link(os.path.join(src_out, O.layer_filename(l)), os.path.join(out, O.layer_filename(l)))
    with open(os.path.join(out, O.layer_filename(5) + ".partial"), "wb") as f:
        f.write(b"interrupted")
    ck = {"completedLayers": m["layers"][:5], "schemaVersion": 2, "sourceIndexSHA256": m["sourceIndexSHA256"]}
    with open(os.path.join(out, "pack.resume.json"), "w") as f:
        json.dump(ck, f)
    with pytest.raises(QfError, match="resume"):
        S.pack_store(d, out)
    r = S.pack_store(d, out, resume=True)
    assert r["layers_written"] == 35
    m2 = json.load(open(os.path.join(out, "manifest.json")))
    assert m2["layers"] == m["layers"]
    assert not os.path.exists(os.path.join(out, "pack.resume.json"))
    assert not os.path.exists(os.path.join(out, O.layer_filename(5) + ".partial"))


def test_a_changed_source_index_is_refused(packed, tmp_path):
    d, _, _ = packed
    c = str(tmp_path / "ck")
    os.makedirs(c)
    for name in os.listdir(d):
        if name.endswith(".safetensors"):
            os.link(os.path.join(d, name), os.path.join(c, name))
    os.symlink(os.path.join(d, "qwen_q4_experts"), os.path.join(c, "qwen_q4_experts"))
    with open(os.path.join(d, "model.safetensors.index.json")) as f, \
            open(os.path.join(c, "model.safetensors.index.json"), "w") as g:
        g.write(f.read() + "\n")
    with pytest.raises(QfError, match="source mismatch"):
        S.pack_store(c)
    with pytest.raises(QfError, match="source mismatch"):
        S.verify_store(c)


def test_pack_refuses_a_checkpoint_without_every_expert_tensor(tmp_path):
    """Discovery fails before any layer is written (the builder's
    discoverSlices: every layer's nine switch_mlp tensors must exist)."""
    d = str(tmp_path / "ck")
    tensors = {}
    for layer in range(40):
        pre = f"language_model.model.layers.{layer}.mlp.switch_mlp."
        for suffix, n, shape, is16 in O.COMPONENTS:
            if layer == 17 and suffix == "down_proj.biases":
                continue
            tensors[pre + suffix] = ("F16" if is16 else "U32", (256,) + shape, O.Sparse(256 * n, {}))
    O.write_checkpoint(d, tensors, n_shards=2)
    with pytest.raises(QfError, match="layers.17.mlp.switch_mlp.down_proj.biases"):
        S.pack_store(d)
    out = os.path.join(d, "qwen_q4_experts")
    assert not any(name.endswith(".q4exp") for name in os.listdir(out))
    with pytest.raises(QfError, match="resume"):  # the progress file it left behind
        S.pack_store(d)
