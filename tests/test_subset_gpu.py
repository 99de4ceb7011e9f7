"""The streaming runner's MoE step as separate entries (qf_shared_expert,
qf_moe_routed_subset for the hit and the miss positions, qf_moe_combine) and
the routed grouped FFN (qf_moe_grouped_ffn), against the CPU oracle and the
whole-block entry.

Reference: QwenQ4ActiveExpertStreamingRunner.swift:1227-1381 dispatches the
shared expert and the hit subset right after planning, then the miss subset
and qwen_combine_cached_moe_subsets_f32 after the reads
(deltanet.metal:2050-2227).  Bar: outputs within max|y - y_ref| / max|y_ref|
<= 2e-3 (fp32 accumulation)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3
SEED, LAYER = 9, 2


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def f32(v):
    return np.float32(v)


def oracle_subset(ys, w, positions):
    """sum over i < 8 of (i < n ? y[p_i] * w[p_i] : 0), left to right, fp32."""
    acc = np.zeros(2048, np.float32)
    parts = [(ys[p] * f32(w[p])).astype(np.float32) if i < len(positions) else np.zeros(2048, np.float32)
             for i, p in enumerate(list(positions) + [0] * (8 - len(positions)))]
    acc = parts[0]
    for q in parts[1:]:
        acc = (acc + q).astype(np.float32)
    return acc


@pytest.fixture(scope="module")
def layer(ctx):
    from qfmoe import MoELayerWeights
    return MoELayerWeights.synth(ctx, SEED, LAYER)


@pytest.fixture(scope="module")
def olayer():
    return O.OracleLayer.synth(SEED, LAYER)


def arena_layer(layer, experts, rng):
    """The layer with its routed records copied into a slot arena at shuffled
    slots; returns (arena layer, slot of each expert)."""
    from qfmoe import MoELayerWeights
    n = len(experts) + 5
    slots = rng.permutation(n)[:len(experts)]
    arena = torch.zeros((n, layer.bank.shape[1]), dtype=torch.uint8, device="cuda")
    for e, s in zip(experts, slots):
        arena[s] = layer.bank[e]
    La = MoELayerWeights(layer.router_w, layer.router_s, layer.router_b, layer.coef_w, layer.coef_s,
                         layer.coef_b, layer.shared, arena)
    return La, dict(zip([int(e) for e in experts], [int(s) for s in slots]))


@pytest.mark.parametrize("hits", [[0, 2, 5], [7, 1], list(range(8)), []],
                         ids=["3hits", "2hits_reordered", "all_hits", "all_misses"])
def test_hit_and_miss_subsets_equal_the_block(ctx, layer, olayer, hits):
    from qfmoe import block_forward, combine, routed_subset, router_logits, router_topk, shared_expert
    from qfmoe import synth_hidden
    rng = np.random.default_rng(len(hits))
    x = synth_hidden(SEED, 40 + len(hits), 1)
    xd = x.cuda()
    res = torch.randn((1, 2048), generator=torch.Generator().manual_seed(3)).cuda()
    logits, coef = router_logits(ctx, layer, xd)
    idx, w = router_topk(ctx, logits)
    e8 = idx[0].cpu().numpy()
    La, slot_of = arena_layer(layer, e8, rng)
    slot_of_pos = torch.tensor([slot_of[int(e)] for e in e8], dtype=torch.int32, device="cuda")
    misses = [p for p in range(8) if p not in hits][::-1]  # any order: the sum follows the list
    sh = shared_expert(ctx, La, xd, coef)
    hit = routed_subset(ctx, La, xd, slot_of_pos, w[0], hits) if hits else None
    miss = routed_subset(ctx, La, xd, slot_of_pos, w[0], misses) if misses else None
    out = combine(ctx, sh, res, hit, miss)
    ctx.check()
    # the CPU oracle's experts in the reference order, combined as the reference does
    x16 = x.numpy().view(np.uint16)
    ref = O.block(olayer, x16, residual=res.cpu().numpy(), threads=8)
    assert np.array_equal(e8, ref["idx"][0])
    ys = {p: O.expert_ffn(O.synth_record(SEED, LAYER, int(e8[p])), x16[0]) for p in range(8)}
    wn = w[0].cpu().numpy()
    c = f32(ref["coef"][0])
    coeff = f32(1.0) / (f32(1.0) + np.exp(-c, dtype=np.float32))
    o_sh = (O.expert_ffn(O.synth_record(SEED, LAYER, 256), x16[0]) * coeff).astype(np.float32)
    o_hit = oracle_subset(ys, wn, hits)
    o_miss = oracle_subset(ys, wn, misses)
    o_out = ((res.cpu().numpy()[0] + o_sh).astype(np.float32) + o_hit).astype(np.float32) + o_miss
    assert max_rel(sh.cpu().numpy()[0], o_sh) < TOL
    if hit is not None:
        assert max_rel(hit.cpu().numpy()[0], o_hit) < TOL
    if miss is not None:
        assert max_rel(miss.cpu().numpy()[0], o_miss) < TOL
    got = out.cpu().numpy()
    assert max_rel(got - res.cpu().numpy(), o_out - res.cpu().numpy()[0]) < TOL
    assert max_rel(got - res.cpu().numpy(), ref["out"] - res.cpu().numpy()) < TOL
    full = block_forward(ctx, layer, xd, res)
    assert max_rel(got - res.cpu().numpy(), (full - res).cpu().numpy()) < TOL


def test_subset_argument_errors_and_bad_slot(ctx, layer):
    import ctypes as C
    from qfmoe import QfError, routed_subset, shared_expert, synth_hidden
    from qfmoe._lib import lib
    xd = synth_hidden(SEED, 0, 1).cuda()
    w = torch.full((8,), 0.125, device="cuda")
    slots = torch.arange(8, dtype=torch.int32, device="cuda")
    out = torch.empty((1, 2048), device="cuda")
    ws = ctx.workspace(1)
    d = layer.desc()
    pos = torch.arange(8, dtype=torch.int32, device="cuda")
    assert lib().qf_moe_routed_subset(ctx.h, C.byref(d), C.c_void_p(xd.data_ptr()),
                                      C.c_void_p(slots.data_ptr()), C.c_void_p(w.data_ptr()),
                                      C.c_void_p(pos.data_ptr()), 9, C.c_void_p(out.data_ptr()),
                                      C.c_void_p(ws.data_ptr()), ws.numel()) == -1
    with pytest.raises(QfError):
        shared_expert(ctx, layer, synth_hidden(SEED, 0, 65).cuda(), torch.zeros(65, device="cuda"))
    # a slot outside the bank is reported on the device, not followed
    bad = slots.clone()
    bad[3] = 10_000
    routed_subset(ctx, layer, xd, bad, w, [3])
    with pytest.raises(QfError, match="QF_ERR_DEVICE"):
        ctx.check()
    ctx.check()


@pytest.mark.parametrize("T", [100, 1])
def test_grouped_ffn_rows_match_the_oracle_experts(ctx, layer, olayer, T):
    from qfmoe import block_forward, grouped_ffn, router_logits, router_topk, shared_expert, synth_hidden
    x = synth_hidden(SEED, 700, T)
    xd = x.cuda()
    logits, coef = router_logits(ctx, layer, xd)
    idx, w = router_topk(ctx, logits)
    y = grouped_ffn(ctx, layer, xd, idx)
    ctx.check()
    x16 = x.numpy().view(np.uint16)
    idx_np = idx.cpu().numpy()
    rng = np.random.default_rng(T)
    for pos in rng.choice(T * 8, min(12, T * 8), replace=False):
        t, k = divmod(int(pos), 8)
        ref = O.expert_ffn(O.synth_record(SEED, LAYER, int(idx_np[t, k])), x16[t])
        assert max_rel(y[pos].cpu().numpy(), ref) < TOL, (t, k)
    # the routed rows, weighted in router order, plus the shared expert: the block
    if T <= 64:
        sh = shared_expert(ctx, layer, xd, coef)
        routed = (y.view(T, 8, 2048) * w.view(T, 8, 1)).sum(1)
        full = block_forward(ctx, layer, xd)
        assert max_rel((routed + sh).cpu().numpy(), full.cpu().numpy()) < TOL
