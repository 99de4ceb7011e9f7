"""MLX checkpoint loader (qf_checkpoint_*): one layer's MoE tensors read from
safetensors shards through the index's weight_map into the host layout of
qf_moe_layer, against the tensors the Python restatement (oracle/store_v2.py)
wrote.  Shards are sparse files: the routed experts that are not given read
as zeros.  No GPU is used."""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import store_v2 as O  # noqa: E402

from qfmoe import QfError  # noqa: E402
from qfmoe.store import Checkpoint  # noqa: E402


def _rand(rng, n):
    return rng.integers(0, 256, n, dtype=np.uint8).tobytes()


def _layer(seed, layer, experts, dtype):
    rng = np.random.default_rng(seed)
    parts = dict(router_w=_rand(rng, 256 * 2048), router_s=_rand(rng, 256 * 64), router_b=_rand(rng, 256 * 64),
                 coef_w=_rand(rng, 2048), coef_s=_rand(rng, 64), coef_b=_rand(rng, 64),
                 shared=_rand(rng, O.RECORD_BYTES))
    bank = {e: _rand(rng, O.RECORD_BYTES) for e in experts}
    t = O.moe_layer_tensors(layer, parts["router_w"], parts["router_s"], parts["router_b"], parts["coef_w"],
                            parts["coef_s"], parts["coef_b"], parts["shared"], bank, dtype)
    return parts, bank, t


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("qwen35b_mlx_4bit"))
    p17, b17, t17 = _layer(1, 17, (0, 5, 255), "BF16")
    p3, b3, t3 = _layer(2, 3, (9,), "F16")
    O.write_checkpoint(d, {**t17, **t3}, n_shards=3)
    return d, {17: (p17, b17), 3: (p3, b3)}


@pytest.mark.parametrize("layer,dtype", [(17, "bf16"), (3, "f16")])
def test_load_layer_matches_the_written_tensors(ckpt, layer, dtype):
    d, want = ckpt
    parts, bank = want[layer]
    with Checkpoint(d) as c:
        got, dt = c.load_layer(layer, threads=4)
    assert dt == dtype
    for k in ("router_w", "router_s", "router_b", "coef_w", "coef_s", "coef_b", "shared"):
        assert got[k].tobytes() == parts[k], k
    for e in range(256):
        row = got["bank"][e]
        if e in bank:
            assert row.tobytes() == bank[e], e
        else:
            assert not row.any(), e


def test_load_layer_without_the_bank(ckpt):
    d, want = ckpt
    with Checkpoint(d) as c:
        got, _ = c.load_layer(17, with_bank=False)
    assert got["bank"] is None and got["shared"].tobytes() == want[17][0]["shared"]


def _rewrite(src, dst, edit):
    """Copy a checkpoint (index + shards) applying edit(tensors_by_shard, index)."""
    os.makedirs(dst)
    index = json.load(open(os.path.join(src, "model.safetensors.index.json")))
    edit(index, dst)
    with open(os.path.join(dst, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f)
    for sn in set(index["weight_map"].values()):
        if not os.path.exists(os.path.join(dst, sn)) and os.path.exists(os.path.join(src, sn)):
            os.link(os.path.join(src, sn), os.path.join(dst, sn))


def test_missing_tensor_in_the_index(ckpt, tmp_path):
    d, _ = ckpt
    name = "language_model.model.layers.17.mlp.switch_mlp.up_proj.scales"
    _rewrite(d, str(tmp_path / "c"), lambda idx, _: idx["weight_map"].pop(name))
    with Checkpoint(str(tmp_path / "c")) as c:
        with pytest.raises(QfError, match="missing " + name):
            c.load_layer(17)


def test_layer_absent_from_the_checkpoint(ckpt):
    d, _ = ckpt
    with Checkpoint(d) as c:
        with pytest.raises(QfError, match="QF_ERR_ARG"):
            c.load_layer(5)
        with pytest.raises(QfError, match="QF_ERR_ARG"):
            c.load_layer(40)


@pytest.mark.parametrize("fault", ["size", "dtype", "mixed"])
def test_bad_tensors_are_rejected(tmp_path, fault):
    parts, bank, t = _layer(3, 0, (1,), "BF16")
    pre = "language_model.model.layers.0.mlp."
    if fault == "size":
        dt, shape, data = t[pre + "gate.scales"]
        t[pre + "gate.scales"] = (dt, shape, data[:-2])
        match = "unexpected byte length"
    elif fault == "dtype":
        dt, shape, data = t[pre + "shared_expert.up_proj.biases"]
        t[pre + "shared_expert.up_proj.biases"] = ("F32", shape, data)
        match = "not BF16 or F16"
    else:
        dt, shape, data = t[pre + "switch_mlp.down_proj.scales"]
        t[pre + "switch_mlp.down_proj.scales"] = ("F16", shape, data)
        match = "mixed scale types"
    d = str(tmp_path / "ck")
    O.write_checkpoint(d, t, n_shards=2)
    with Checkpoint(d) as c:
        with pytest.raises(QfError, match=match):
            c.load_layer(0)


def test_bad_index_and_missing_shard(ckpt, tmp_path):
    (tmp_path / "a").mkdir()
    (tmp_path / "a" / "model.safetensors.index.json").write_text('{"metadata": {}}')
    with pytest.raises(QfError, match="weight_map"):
        Checkpoint(str(tmp_path / "a"))
    (tmp_path / "b").mkdir()
    (tmp_path / "b" / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {"x": "../escape.safetensors"}}))
    with pytest.raises(QfError, match="shard name"):
        Checkpoint(str(tmp_path / "b"))
    d, _ = ckpt
    some = json.load(open(os.path.join(d, "model.safetensors.index.json")))["weight_map"]
    shard = sorted(set(some.values()))[0]
    _rewrite(d, str(tmp_path / "c"), lambda idx, dst: None)
    os.remove(str(tmp_path / "c" / shard))
    with Checkpoint(str(tmp_path / "c")) as c:
        with pytest.raises(QfError, match="QF_ERR_IO"):
            c.load_layer(17)
    with pytest.raises(QfError, match="QF_ERR_IO"):
        Checkpoint(str(tmp_path / "nowhere"))


def _open_fds():
    return len(os.listdir("/proc/self/fd"))


def test_bad_shard_header_leaks_no_descriptor(ckpt, tmp_path):
    """A shard whose safetensors header does not parse fails every load with
    QF_ERR_ARG, and each failed open is closed: repeated loads keep the
    process's descriptor count unchanged."""
    d, _ = ckpt
    some = json.load(open(os.path.join(d, "model.safetensors.index.json")))["weight_map"]
    shard = sorted(set(some.values()))[0]

    def corrupt(idx, dst):
        with open(os.path.join(dst, shard), "wb") as f:
            f.write((16).to_bytes(8, "little") + b"not a json head!")

    _rewrite(d, str(tmp_path / "c"), corrupt)
    with Checkpoint(str(tmp_path / "c")) as c:
        with pytest.raises(QfError, match="safetensors header"):
            c.load_layer(17)
        n0 = _open_fds()
        for _ in range(5):
            with pytest.raises(QfError, match="safetensors header"):
                c.load_layer(17)
        assert _open_fds() == n0
