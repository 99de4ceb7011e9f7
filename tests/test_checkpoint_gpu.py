"""A layer loaded from an MLX safetensors checkpoint runs the MoE block bit for
bit like the same weights generated on the device: the synthetic layer is
written as checkpoint tensors (names and shapes of the reference's model,
oracle/store_v2.py), read back by the native loader, uploaded, and both run
through block_forward at batch 1 (one-token kernel) and 16 tokens (grouped
path)."""
import os
import sys

import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import store_v2 as SO  # noqa: E402

pytestmark = pytest.mark.gpu

SEED = 9


def test_checkpoint_layer_equals_synthetic_layer(ctx, tmp_path):
    from qfmoe import RECORD_BYTES, MoELayerWeights, block_forward, synth_hidden
    from qfmoe.store import Checkpoint
    src = MoELayerWeights.synth(ctx, SEED, 11)
    b = lambda t: t.cpu().numpy().tobytes()  # noqa: E731
    bank = src.bank.cpu().numpy()
    tensors = SO.moe_layer_tensors(11, b(src.router_w), b(src.router_s), b(src.router_b), b(src.coef_w),
                                   b(src.coef_s), b(src.coef_b), b(src.shared),
                                   {e: bank[e, :RECORD_BYTES].tobytes() for e in range(256)}, "F16")
    d = str(tmp_path / "ckpt")
    SO.write_checkpoint(d, tensors, n_shards=2)
    with Checkpoint(d) as c:
        layer, dtype = c.layer_weights(ctx, 11)
    assert dtype == "f16"
    for T in (1, 16):
        x = synth_hidden(SEED, 0, T).cuda()
        got = block_forward(ctx, layer, x)
        want = block_forward(ctx, src, x)
        ctx.check()
        assert torch.equal(got, want), T
