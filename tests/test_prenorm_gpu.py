"""The MoE block from the residual stream (qf_moe_block_forward_prenorm): the
post-attention RMSNorm kernel gives the same fp16 input as the CPU oracle's
restatement of qwen_rmsnorm_f32 (64 threads, fma chains, lane butterfly),
so the block output equals block_forward on the oracle's input with the
stream as residual, bit for bit, on the one-token kernel (T = 1), the
persistent batch kernel (T = 3) and the grouped path (T = 16)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 3, 16])
def test_prenorm_block_equals_block_on_oracle_norm(ctx, T):
    from qfmoe import MoELayerWeights, block_forward, block_forward_prenorm
    layer = MoELayerWeights.synth(ctx, 4, 2)
    rng = np.random.default_rng(T)
    h = (rng.standard_normal((T, 2048)) * 3.0).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    hd, wd = torch.from_numpy(h).cuda(), torch.from_numpy(w).cuda()
    got, idx, _ = block_forward_prenorm(ctx, layer, hd, wd, 1e-6, return_routing=True)
    x16 = torch.from_numpy(O.post_norm_f16(h, w, 1e-6).view(np.int16).reshape(T, 2048)).cuda().view(torch.float16)
    want, idx2, _ = block_forward(ctx, layer, x16, hd, return_routing=True)
    ctx.check()
    assert torch.equal(idx, idx2)
    assert torch.equal(got, want)
