"""GPU parity of the decode-path MoE block against the CPU oracle.

Bar: expert indices bit-exact (ties to the lower index);
outputs within max|y - y_ref| / max|y_ref| <= 2e-3 with fp32 accumulation.
Router logits are bit-exact: the kernel uses the reference lane order
(deltanet.metal:2229-2260) and the oracle reproduces its butterfly.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3
SEED = 0


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="module")
def layers(ctx):
    from qfmoe import MoELayerWeights
    return {
        (0, False): MoELayerWeights.synth(ctx, SEED, 0),
        (1, False): MoELayerWeights.synth(ctx, SEED, 1),
    }


@pytest.fixture(scope="module")
def oracle_layers():
    return {0: O.OracleLayer.synth(SEED, 0), 1: O.OracleLayer.synth(SEED, 1)}


def hidden(T, tok0=0):
    from qfmoe import synth_hidden
    return synth_hidden(SEED, tok0, T)


def test_synth_bytes_match_oracle(ctx, layers):
    L = layers[(0, False)]
    torch.cuda.synchronize()
    w, s, b = O.synth_router(SEED, 0)
    assert np.array_equal(L.router_w.cpu().numpy(), w)
    assert np.array_equal(L.router_s.cpu().numpy().view(np.uint16), s)
    assert np.array_equal(L.router_b.cpu().numpy().view(np.uint16), b)
    cw, cs, cb = O.synth_coef(SEED, 0)
    assert np.array_equal(L.coef_w.cpu().numpy(), cw)
    assert np.array_equal(L.coef_s.cpu().numpy().view(np.uint16), cs)
    assert np.array_equal(L.shared.cpu().numpy(), O.synth_record(SEED, 0, 256))
    for e in (0, 77, 255):
        assert np.array_equal(L.bank[e].cpu().numpy(), O.synth_record(SEED, 0, e)), e
    x = hidden(3, tok0=5)
    assert np.array_equal(x.numpy().view(np.uint16), O.synth_hidden(SEED, 5, 3))


def test_synth_bf16_bytes_match_oracle():
    from qfmoe import MoEContext, MoELayerWeights, synth_records
    c = MoEContext(0, scale_bf16=True)
    rec = torch.empty((2, O.RECORD_BYTES), dtype=torch.uint8, device="cuda")
    synth_records(c, 3, 7, 100, 2, rec)
    torch.cuda.synchronize()
    for i in range(2):
        assert np.array_equal(rec[i].cpu().numpy(), O.synth_record(3, 7, 100 + i, bf16=True))
    L = MoELayerWeights.synth(c, 3, 7, n_records=1)
    torch.cuda.synchronize()
    assert np.array_equal(L.router_s.cpu().numpy().view(np.uint16), O.synth_router(3, 7, True)[1])


@pytest.mark.parametrize("T", [1, 5, 64])
def test_router_logits_bitexact(ctx, layers, oracle_layers, T):
    from qfmoe import router_logits
    x = hidden(T, tok0=11)
    logits, coef = router_logits(ctx, layers[(0, False)], x.cuda())
    ref = O.block(oracle_layers[0], x.numpy().view(np.uint16), threads=8)
    got = logits.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref["logits"].view(np.uint32))
    assert max_rel(coef.cpu().numpy(), ref["coef"]) < 1e-5


def test_topk_matches_oracle_and_breaks_ties_low(ctx):
    from qfmoe import router_topk
    rng = np.random.default_rng(1)
    T = 40
    logits = rng.standard_normal((T, 256)).astype(np.float32)
    # ties: duplicate values at several indices, including across the top-8 boundary
    logits[0, :] = 0.0
    logits[1, [3, 9, 200, 201, 17]] = 5.0
    logits[2, ::2] = 1.0
    logits[3, 250:] = 7.0
    bias = rng.standard_normal(256).astype(np.float32) * 0.1
    for b in (None, bias):
        idx, w = router_topk(ctx, torch.from_numpy(logits).cuda(),
                             None if b is None else torch.from_numpy(b).cuda())
        ridx, rw = O.topk(logits, 8, b)
        assert np.array_equal(idx.cpu().numpy(), ridx)
        assert max_rel(w.cpu().numpy(), rw) < 1e-5
        if b is None:
            got = idx.cpu().numpy()
            assert got[0].tolist() == list(range(8))
            assert got[1][:5].tolist() == [3, 9, 17, 200, 201]
            assert got[3].tolist() == list(range(250, 256)) + got[3][6:].tolist()


@pytest.mark.parametrize("T", [1, 3, 8, 33, 64])
def test_block_parity(ctx, layers, oracle_layers, T):
    from qfmoe import block_forward
    x = hidden(T, tok0=100 + T)
    out, idx, w = block_forward(ctx, layers[(0, False)], x.cuda(), return_routing=True)
    ctx.check()
    ref = O.block(oracle_layers[0], x.numpy().view(np.uint16), threads=8)
    assert np.array_equal(idx.cpu().numpy(), ref["idx"])
    assert max_rel(w.cpu().numpy(), ref["w"]) < 1e-5
    err = max_rel(out.cpu().numpy(), ref["out"])
    assert err < TOL, err


def test_block_residual_and_determinism(ctx, layers, oracle_layers):
    from qfmoe import block_forward
    T = 4
    x = hidden(T, tok0=7)
    res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(3)).float()
    o1 = block_forward(ctx, layers[(0, False)], x.cuda(), res.cuda())
    o2 = block_forward(ctx, layers[(0, False)], x.cuda(), res.cuda())
    assert torch.equal(o1, o2)  # bitwise run-to-run determinism
    ref = O.block(oracle_layers[0], x.numpy().view(np.uint16), residual=res.numpy(), threads=8)
    assert max_rel(o1.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T", [1, 6, 20])
def test_block_supplied_routing_and_slot_table(ctx, layers, oracle_layers, T):
    """Routing supplied by the oracle; records addressed through a permuted slot arena
    (the cache's slot_indices, deltanet.metal:2155-2211).  T = 1 runs the one-token
    kernel, T = 6 the T <= 8 persistent kernel, T = 20 the per-kernel decode path
    (a slot arena keeps T = 9..64 off the grouped path)."""
    from qfmoe import block_forward
    x = hidden(T, tok0=300)
    rng = np.random.default_rng(5)
    idx = np.stack([rng.choice(256, 8, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, 8)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    ref = O.block(oracle_layers[0], x.numpy().view(np.uint16), idx_in=idx, w_in=w, threads=8)
    L = layers[(0, False)]
    # arena with the needed records at shuffled slots
    uniq = np.unique(idx)
    slots = rng.permutation(len(uniq) + 5)[: len(uniq)]
    arena = torch.zeros((len(uniq) + 5, L.bank.shape[1]), dtype=torch.uint8, device="cuda")
    for e, s in zip(uniq, slots):
        arena[s] = L.bank[e]
    slot_of = dict(zip(uniq.tolist(), slots.tolist()))
    rec = np.vectorize(slot_of.get)(idx).astype(np.int32)
    from qfmoe import MoELayerWeights
    La = MoELayerWeights(L.router_w, L.router_s, L.router_b, L.coef_w, L.coef_s, L.coef_b,
                         L.shared, arena)
    out, gi, gw = block_forward(ctx, La, x.cuda(), topk_idx=torch.from_numpy(idx).cuda(),
                                topk_w=torch.from_numpy(w).cuda(),
                                record_of_pos=torch.from_numpy(rec).cuda(), return_routing=True)
    ctx.check()
    assert np.array_equal(gi.cpu().numpy(), idx)
    assert max_rel(out.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T", [1, 3])
def test_block_router_ties_go_to_the_lower_index(ctx, layers, T):
    """Exact logit ties through the whole block: router rows duplicated so that a
    lower-index copy of token 0's top expert ties with it (it must rank just
    before it) and a higher-index copy of the 8th expert ties with that one (it
    must lose the last place), as the reference's strict-> scan orders them
    (deltanet.metal:2283-2329).  T = 1 runs the one-token kernel's top-8."""
    from qfmoe import MoELayerWeights, block_forward
    x = hidden(T, tok0=31)
    rw, rs, rb = (a.copy() for a in O.synth_router(SEED, 0))
    coef = O.synth_coef(SEED, 0)
    shared = O.synth_record(SEED, 0, 256)
    lg, _ = O.router(O.OracleLayer((rw, rs, rb), coef, shared, {}), x.numpy().view(np.uint16)[:1])
    order = [int(e) for e in np.argsort(-lg[0], kind="stable")]
    top = order[0]
    lo = next((e for e in range(top) if e not in order[:8]), None)
    # the expert that ranks 8th once the copy of the top expert takes a place
    eighth = order[6] if lo is not None else order[7]
    hi = next(e for e in range(eighth + 1, 256) if e not in order[:8])
    W, S, B = rw.reshape(256, -1), rs.reshape(256, -1), rb.reshape(256, -1)
    for src, dst in ([(top, lo)] if lo is not None else []) + [(eighth, hi)]:
        W[dst], S[dst], B[dst] = W[src], S[src], B[src]
    OL = O.OracleLayer((rw, rs, rb), coef, shared, {e: O.synth_record(SEED, 0, e) for e in range(256)})
    ref = O.block(OL, x.numpy().view(np.uint16), threads=8)
    if lo is not None:
        assert list(ref["idx"][0, :2]) == [lo, top]
    assert hi not in ref["idx"][0] and eighth in ref["idx"][0]
    L = layers[(0, False)]
    Lt = MoELayerWeights(torch.from_numpy(rw).cuda(), torch.from_numpy(rs.view(np.int16)).cuda(),
                         torch.from_numpy(rb.view(np.int16)).cuda(), L.coef_w, L.coef_s, L.coef_b,
                         L.shared, L.bank)
    out, idx, _ = block_forward(ctx, Lt, x.cuda(), return_routing=True)
    ctx.check()
    assert np.array_equal(idx.cpu().numpy(), ref["idx"])
    assert max_rel(out.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T", [1, 16])
def test_block_logit_bias(ctx, layers, oracle_layers, T):
    from qfmoe import block_forward
    x = hidden(T, tok0=900)
    bias = (np.log(1.0 / np.arange(1, 257) ** 1.1) * 2.0).astype(np.float32)
    out, idx, _ = block_forward(ctx, layers[(0, False)], x.cuda(),
                                logit_bias=torch.from_numpy(bias).cuda(), return_routing=True)
    ref = O.block(oracle_layers[0], x.numpy().view(np.uint16), bias=bias, threads=8)
    assert np.array_equal(idx.cpu().numpy(), ref["idx"])
    assert max_rel(out.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T", [1, 2])
def test_block_bf16_scales(T):
    from qfmoe import MoEContext, MoELayerWeights, block_forward
    c = MoEContext(0, scale_bf16=True)
    L = MoELayerWeights.synth(c, 9, 2)
    OL = O.OracleLayer.synth(9, 2, bf16=True)
    x = hidden(T, tok0=50)
    out, idx, _ = block_forward(c, L, x.cuda(), return_routing=True)
    ref = O.block(OL, x.numpy().view(np.uint16), threads=8)
    assert np.array_equal(idx.cpu().numpy(), ref["idx"])
    assert max_rel(out.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T", [1, 3, 12])
def test_stack_equals_chained_blocks_with_oracle_norm(ctx, layers, oracle_layers, T):
    """Two stacked blocks == block 0, the oracle's RMSNorm of its output, block 1:
    bitwise, which pins the in-kernel RMSNorm (deltanet.metal:18-53) to the oracle.
    T = 1 runs the one-token persistent kernel, T = 3 the T <= 8 persistent
    kernel, T = 12 the grouped tcgen05 path with the RMSNorm kernel between
    blocks."""
    from qfmoe import StackPlan, block_forward, stack_forward
    x = hidden(T, tok0=40)
    plan = StackPlan([layers[(0, False)], layers[(1, False)]])
    out, idx, _ = stack_forward(ctx, plan, x.cuda(), eps=1e-6, return_routing=True)
    h1 = block_forward(ctx, layers[(0, False)], x.cuda())
    x1 = O.rmsnorm_to_f16(h1.cpu().numpy(), 1e-6)
    x1t = torch.from_numpy(x1.view(np.float16)).cuda()
    h2, idx1, _ = block_forward(ctx, layers[(1, False)], x1t, h1, return_routing=True)
    assert torch.equal(out, h2)
    assert torch.equal(idx[1], idx1)
    # and layer 1 against the oracle on the same inputs
    ref = O.block(oracle_layers[1], x1, residual=h1.cpu().numpy(), threads=8)
    assert np.array_equal(idx1.cpu().numpy(), ref["idx"])
    assert max_rel(h2.cpu().numpy() - h1.cpu().numpy(), ref["out"] - h1.cpu().numpy()) < TOL


def test_bad_record_is_reported_not_faulted(ctx, layers):
    from qfmoe import QfError, block_forward
    x = hidden(1)
    idx = torch.arange(8, dtype=torch.int32, device="cuda").view(1, 8)
    w = torch.full((1, 8), 0.125, device="cuda")
    rec = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 10_000]], dtype=torch.int32, device="cuda")
    block_forward(ctx, layers[(0, False)], x.cuda(), topk_idx=idx, topk_w=w, record_of_pos=rec)
    with pytest.raises(QfError, match="QF_ERR_DEVICE"):
        ctx.check()
    ctx.check()  # status word cleared


def test_argument_errors(ctx, layers):
    import ctypes as C
    from qfmoe._lib import lib
    x = hidden(8).cuda()
    out = torch.empty((8, 2048), device="cuda")
    ws = ctx.workspace(8)
    d = layers[(0, False)].desc()
    f = lib().qf_moe_block_forward
    args = (x.data_ptr(), None, out.data_ptr(), None, None, None, ws.data_ptr(), ws.numel())
    assert f(ctx.h, C.byref(d), 40000, *args) == -1  # T above the prefill limit
    assert f(ctx.h, C.byref(d), 0, *args) == -1
    d.expert_bank += 16  # records are read 32 bytes at a time
    assert f(ctx.h, C.byref(d), 8, *args) == -1
    d = layers[(0, False)].desc()
    d.record_stride += 16
    assert f(ctx.h, C.byref(d), 8, *args) == -1
    torch.cuda.synchronize()


def test_dispatch_plan_matches_oracle(ctx):
    from qfmoe import dispatch_plan
    rng = np.random.default_rng(7)
    for T in (1, 37, 4096):
        p = 1.0 / np.arange(1, 257) ** 1.1
        p /= p.sum()
        idx = np.stack([rng.choice(256, 8, replace=False, p=p) for _ in range(T)]).astype(np.int32)
        c, o, perm = dispatch_plan(ctx, torch.from_numpy(idx).cuda())
        rc, ro, rp = O.dispatch_plan(idx)
        assert np.array_equal(c.cpu().numpy(), rc)
        assert np.array_equal(o.cpu().numpy(), ro)
        assert np.array_equal(perm.cpu().numpy(), rp)


@pytest.mark.parametrize("T", [1, 8])
def test_persistent_and_per_kernel_paths_agree(ctx, layers, oracle_layers, T):
    """T <= 8 runs the persistent kernel; with per-kernel timing enabled the same
    call runs the five-kernel path.  Both must meet the oracle bar."""
    from qfmoe import block_forward, profile_begin, profile_end
    x = hidden(T, tok0=700)
    o1, i1, _ = block_forward(ctx, layers[(1, False)], x.cuda(), return_routing=True)
    profile_begin(ctx, "gate_up", 16)
    o2, i2, _ = block_forward(ctx, layers[(1, False)], x.cuda(), return_routing=True)
    ms, n = profile_end(ctx)
    assert n == 1 and ms > 0
    ref = O.block(oracle_layers[1], x.numpy().view(np.uint16), threads=8)
    assert np.array_equal(i1.cpu().numpy(), ref["idx"])
    assert np.array_equal(i2.cpu().numpy(), ref["idx"])
    assert max_rel(o1.cpu().numpy(), ref["out"]) < TOL
    assert max_rel(o2.cpu().numpy(), ref["out"]) < TOL


@pytest.mark.parametrize("T,n_layers", [(2, 5), (1, 5), (1, 67)])
def test_stack_long_chain_matches_blocks(ctx, layers, T, n_layers):
    """A stack of alternating layers 0,1,0,... equals the chain of single blocks with
    the in-kernel norm emulated by the oracle, bitwise.  67 layers at T = 1 cross
    the 64-layer split of the persistent launch."""
    from qfmoe import StackPlan, block_forward, stack_forward
    x = hidden(T, tok0=77)
    seq = [layers[(l % 2, False)] for l in range(n_layers)]
    out = stack_forward(ctx, StackPlan(seq), x.cuda(), eps=1e-6)
    h = block_forward(ctx, seq[0], x.cuda())
    for L in seq[1:]:
        xn = torch.from_numpy(O.rmsnorm_to_f16(h.cpu().numpy(), 1e-6).view(np.float16)).cuda()
        h = block_forward(ctx, L, xn, h)
    assert torch.equal(out, h)
