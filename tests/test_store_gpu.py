"""Packed expert store as the source of the host tier, end to end on the GPU:
a layer's records written in the reference's v2 format (by the restatement
oracle/store_v2.py), loaded by the native reader into pinned host memory,
copied into HBM slots by the tier, and read by the decode kernel through the
slot map give results bitwise equal to the resident bank."""
import hashlib
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import store_v2 as SO  # noqa: E402

pytestmark = pytest.mark.gpu

SEED = 5


def test_store_to_tier_to_slots_matches_resident(ctx, tmp_path):
    from qfmoe import RECORD_BYTES, MoELayerWeights, block_forward, synth_hidden
    from qfmoe.cache import ArenaLayer, HostTier
    from qfmoe.store import ExpertStore
    layer = MoELayerWeights.synth(ctx, SEED, 0)
    bank = layer.bank.cpu().numpy()  # [256, RECORD_BYTES] (+ stride padding)
    records = {(6, e): bank[e, :RECORD_BYTES].tobytes() for e in range(256)}
    index = tmp_path / "model.safetensors.index.json"
    index.write_text('{"weight_map": {"synthetic": "seed %d"}}\n' % SEED)
    d = str(tmp_path / "qwen_q4_experts")
    SO.write_store(d, hashlib.sha256(index.read_bytes()).hexdigest(), records, hash_layers=(6,))

    host = torch.empty((256, RECORD_BYTES), dtype=torch.uint8, pin_memory=True)
    with ExpertStore(d, str(index)) as s:
        assert s.verify_layer(6)
        s.load_tier(host, first_layer=6, n_layers=1)
        assert s.metrics()["packed_reads"] == 256
    assert np.array_equal(host.numpy(), bank[:, :RECORD_BYTES])

    tier = HostTier(0, 16, host)
    rng = np.random.default_rng(SEED)
    x = synth_hidden(SEED, 0, 1).cuda()
    for t in range(3):
        experts = rng.choice(256, 8, replace=False).astype(np.int32)
        slots = np.arange(8, dtype=np.uint32) + 8 * (t % 2)
        tier.fetch(experts, slots)
        ti = torch.from_numpy(experts[None].copy()).cuda()
        w = rng.random(8).astype(np.float32)
        tw = torch.from_numpy((w / w.sum())[None]).cuda()
        rec = torch.from_numpy(slots.astype(np.int32)[None].copy()).cuda()
        got = block_forward(ctx, ArenaLayer(layer, tier), x, topk_idx=ti, topk_w=tw, record_of_pos=rec)
        want = block_forward(ctx, layer, x, topk_idx=ti, topk_w=tw)
        ctx.check()
        assert torch.equal(got, want), t
    tier.close()
