"""Q4 LM head (qf_lm_head_q4) against the CPU oracle's restatement of the
reference GEMV (qwen_gemv_q4_affine_simd_f32 over qwen_q4_row_simd_f32,
deltanet.metal:1838-1919): logits equal bit for bit, at the full 248,320-row
vocabulary and at ragged row counts, with fp16 and bf16 scales, one and two
token rows.  Weights follow the benchmark's synthetic distribution: codes
uniform 0..15, scale |N(0, 0.01)| + 1e-3, bias -8 * scale; x an RMS-normalised
N(0, 1) row."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

VOCAB = 248_320


def weights(rows, bf16, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, (rows, 1024), dtype=np.uint8)
    s = np.abs(rng.normal(0.0, 0.01, (rows, 32))) + 1e-3
    b = -8.0 * s
    if bf16:
        cvt = lambda a: (torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy())  # noqa: E731
    else:
        cvt = lambda a: a.astype(np.float16).view(np.int16)  # noqa: E731
    return w, cvt(s), cvt(b)


def xrow(seed, T=1):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, 2048)).astype(np.float32)
    return (x / np.sqrt(np.mean(x * x, axis=1, keepdims=True))).astype(np.float32)


@pytest.mark.parametrize("bf16", [False, True])
def test_lm_head_full_vocab_bitwise(bf16):
    from qfmoe import MoEContext, lm_head
    ctx = MoEContext(0, scale_bf16=bf16)
    w, s, b = weights(VOCAB, bf16, 7 + bf16)
    x = xrow(3)
    got = lm_head(ctx, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(b).cuda(),
                  torch.from_numpy(x).cuda())
    ctx.check()
    ref = O.lm_head(w, s.view(np.uint16), b.view(np.uint16), x[0], bf16=bf16)
    g = got.cpu().numpy()[0]
    assert np.array_equal(g.view(np.uint32), ref.view(np.uint32)), np.flatnonzero(g != ref)[:10]
    assert int(np.argmax(g)) == int(np.argmax(ref))


@pytest.mark.parametrize("rows", [1, 7, 1000, 5921])
def test_lm_head_ragged_rows_and_two_tokens(rows):
    from qfmoe import MoEContext, lm_head
    ctx = MoEContext(0)
    w, s, b = weights(rows, False, rows)
    x = xrow(rows, T=2)
    got = lm_head(ctx, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(b).cuda(),
                  torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.check()
    for t in range(2):
        ref = O.lm_head(w, s.view(np.uint16), b.view(np.uint16), x[t])
        assert np.array_equal(got[t].view(np.uint32), ref.view(np.uint32)), (rows, t)


def test_lm_head_argument_errors():
    from qfmoe import MoEContext, QfError, lm_head
    ctx = MoEContext(0)
    w, s, b = (torch.from_numpy(a).cuda() for a in weights(64, False, 1))
    x = torch.from_numpy(xrow(1)).cuda()
    with pytest.raises(QfError):  # x not 16-B aligned
        lm_head(ctx, w, s, b, torch.zeros(2049, device="cuda")[1:])
    with pytest.raises(QfError):  # no rows
        lm_head(ctx, w[:0], s[:0], b[:0], x)
