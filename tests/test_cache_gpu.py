"""Expert-slot cache on the GPU: records copied from the pinned-host tier into
HBM slots are read back through the slot map with results bitwise equal to
the resident bank, and the streaming decode step (plan per layer, copy the
misses on the tier's stream, one persistent kernel per step) equals the
chain of resident blocks with the oracle's RMSNorm between layers."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

SEED = 3
N_LAYERS = 4
TOL = 2e-3


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="module")
def stack(ctx):
    """N_LAYERS resident layers and a pinned host copy of their routed records
    (host record l * 256 + e = expert e of layer l)."""
    from qfmoe import RECORD_BYTES, MoELayerWeights
    layers = [MoELayerWeights.synth(ctx, SEED, l) for l in range(N_LAYERS)]
    host = torch.empty((N_LAYERS * 256, RECORD_BYTES), dtype=torch.uint8, pin_memory=True)
    for l, L in enumerate(layers):
        host[l * 256:(l + 1) * 256].copy_(L.bank)
    torch.cuda.synchronize()
    return layers, host


def trace(n_tokens, seed):
    rng = np.random.default_rng(seed)
    idx = np.zeros((n_tokens, N_LAYERS, 8), np.int32)
    w = rng.random((n_tokens, N_LAYERS, 8)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    hot = rng.permutation(256)[:24]  # a small popular set so slots get reused
    for t in range(n_tokens):
        for l in range(N_LAYERS):
            pool = hot if rng.random() < 0.6 else np.arange(256)
            idx[t, l] = rng.choice(pool, 8, replace=False)
    return idx, w


def test_tier_fetch_then_slot_reads_match_resident(ctx, stack):
    from qfmoe import block_forward, synth_hidden
    from qfmoe.cache import ArenaLayer, ExpertCache, HostTier
    layers, host = stack
    cache = ExpertCache(16, layer_count=1)
    tier = HostTier(0, 16, host)
    x = synth_hidden(SEED, 0, 1).cuda()
    idx, w = trace(6, 11)
    for t in range(6):
        e = idx[t, 0]
        slots, miss, fetch = cache.acquire_slots_parallel(0, e)
        tier.fetch([fe for fe, _ in fetch], [fs for _, fs in fetch])  # layer 0: host index = expert
        ti = torch.from_numpy(e[None].copy()).cuda()
        tw = torch.from_numpy(w[t, 0][None].copy()).cuda()
        rec = torch.tensor([slots], dtype=torch.int32, device="cuda")
        got = block_forward(ctx, ArenaLayer(layers[0], tier), x, topk_idx=ti, topk_w=tw,
                            record_of_pos=rec)
        want = block_forward(ctx, layers[0], x, topk_idx=ti, topk_w=tw)
        ctx.check()
        assert torch.equal(got, want), t
    st = tier.stats()
    m = cache.metrics_snapshot()
    assert st["copies"] == m["misses"] and st["bytes"] == m["fetched_bytes"]
    tier.close()


@pytest.mark.parametrize("capacity,policy", [(N_LAYERS * 10, "slru"), (N_LAYERS * 12, "lru"),
                                             (N_LAYERS * 256, "slru")])
def test_stream_step_equals_resident_chain(ctx, stack, capacity, policy):
    """Steps are enqueued back to back (copies of step n+1 may overlap step n's
    kernel); every step's output equals the resident chain bitwise."""
    from qfmoe import HIDDEN, StackPlan, block_forward, synth_hidden
    from qfmoe.cache import ExpertCache, HostTier, stream_step
    layers, host = stack
    n_tok = 8
    idx, w = trace(n_tok, 7)
    cache = ExpertCache(capacity, layer_count=N_LAYERS, policy=policy)
    tier = HostTier(0, capacity, host)
    plan = StackPlan(layers)
    xs = synth_hidden(SEED, 100, n_tok).cuda()
    outs = torch.empty((n_tok, 1, HIDDEN), dtype=torch.float32, device="cuda")
    ws = ctx.workspace(1)
    for t in range(n_tok):
        stream_step(ctx, cache, tier, plan, idx[t], w[t], xs[t:t + 1], None, outs[t], 1e-6,
                    workspace=ws)
    ctx.check()
    m = cache.metrics_snapshot()
    assert m["hits"] + m["misses"] == n_tok * N_LAYERS * 8
    if capacity < N_LAYERS * 256:
        assert m["evictions"] > 0
    for t in range(n_tok):
        x = xs[t:t + 1]
        h = None
        for l in range(N_LAYERS):
            ti = torch.from_numpy(idx[t, l][None].copy()).cuda()
            tw = torch.from_numpy(w[t, l][None].copy()).cuda()
            h = block_forward(ctx, layers[l], x, h, topk_idx=ti, topk_w=tw)
            if l + 1 < N_LAYERS:
                x = torch.from_numpy(O.rmsnorm_to_f16(h.cpu().numpy(), 1e-6).view(np.float16)).cuda()
        assert torch.equal(outs[t], h), t
    tier.close()


def test_stream_step_first_layer_vs_oracle(ctx, stack):
    """One-layer stream step against the CPU oracle block with the same routing."""
    from qfmoe import HIDDEN, StackPlan, synth_hidden
    from qfmoe.cache import ExpertCache, HostTier, stream_step
    layers, host = stack
    OL = O.OracleLayer.synth(SEED, 0)
    idx, w = trace(2, 21)
    cache = ExpertCache(8, layer_count=1)
    tier = HostTier(0, 8, host)
    plan = StackPlan(layers[:1])
    for t in range(2):
        x = synth_hidden(SEED, 500 + t, 1)
        out = torch.empty((1, HIDDEN), dtype=torch.float32, device="cuda")
        stream_step(ctx, cache, tier, plan, idx[t, :1], w[t, :1], x.cuda(), None, out)
        ctx.check()
        ref = O.block(OL, x.numpy().view(np.uint16), idx_in=idx[t, :1], w_in=w[t, :1], threads=8)
        assert max_rel(out.cpu().numpy(), ref["out"]) < TOL
    tier.close()


def test_stream_step_argument_errors(ctx, stack):
    from qfmoe import HIDDEN, QfError, StackPlan, synth_hidden
    from qfmoe.cache import ExpertCache, HostTier, stream_step
    layers, host = stack
    plan = StackPlan(layers[:2])
    x = synth_hidden(SEED, 0, 1).cuda()
    out = torch.empty((1, HIDDEN), dtype=torch.float32, device="cuda")
    idx = np.zeros((2, 8), np.int32)
    idx[:] = np.arange(8)
    w = np.full((2, 8), 0.125, np.float32)
    tier = HostTier(0, 16, host)
    with pytest.raises(QfError):  # one partition for two layers
        stream_step(ctx, ExpertCache(15, layer_count=2), tier, plan, idx, w, x, None, out)
    with pytest.raises(QfError):  # cache larger than the arena
        stream_step(ctx, ExpertCache(32, layer_count=2), tier, plan, idx, w, x, None, out)
    bad = idx.copy()
    bad[1, 3] = 256
    with pytest.raises(QfError):  # expert id out of range
        stream_step(ctx, ExpertCache(16, layer_count=2), tier, plan, bad, w, x, None, out)
    with pytest.raises(QfError):  # host index beyond the host records
        HostTier(0, 4, host[:10]).fetch([10], [0])
    with pytest.raises(QfError):  # slot beyond the arena
        tier.fetch([0], [16])
    ctx.check()
    tier.close()


def test_stream_step_injected_short_copy(ctx, stack):
    """Host-side fault injection: one record copy of a step is treated as a
    short copy.  The step returns QF_ERR_IO without running, the tier counts
    the failure, the cache does not map the expert whose bytes never arrived,
    and the same step retried equals the resident chain bitwise."""
    from qfmoe import HIDDEN, QfError, StackPlan, block_forward, synth_hidden
    from qfmoe.cache import ExpertCache, HostTier, stream_step
    layers, host = stack
    idx, w = trace(4, 31)
    capacity = N_LAYERS * 10
    cache = ExpertCache(capacity, layer_count=N_LAYERS)
    tier = HostTier(0, capacity, host)
    plan = StackPlan(layers)
    xs = synth_hidden(SEED, 700, 4).cuda()
    out = torch.full((1, HIDDEN), float("nan"), device="cuda")
    ws = ctx.workspace(1)
    for t in range(2):
        stream_step(ctx, cache, tier, plan, idx[t], w[t], xs[t:t + 1], None, out, 1e-6, workspace=ws)
    torch.cuda.synchronize()
    ctx.check()
    m0 = cache.metrics_snapshot()
    s0 = tier.stats()
    assert s0["failed"] == 0
    out.fill_(float("nan"))
    tier.inject_fault(1, 1)  # the second record copy of the next step fails
    with pytest.raises(QfError, match="QF_ERR_IO"):
        stream_step(ctx, cache, tier, plan, idx[2], w[2], xs[2:3], None, out, 1e-6, workspace=ws)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.isnan(out).all()  # the step did not run
    s1 = tier.stats()
    m1 = cache.metrics_snapshot()
    assert s1["failed"] == 1
    misses_2 = m1["misses"] - m0["misses"]
    assert misses_2 >= 2
    assert s1["copies"] - s0["copies"] == misses_2 - 1
    assert m1["fetched_bytes"] - m0["fetched_bytes"] == (misses_2 - 1) * 1_769_472
    # retry: the failed expert misses again and is fetched; output is exact
    stream_step(ctx, cache, tier, plan, idx[2], w[2], xs[2:3], None, out, 1e-6, workspace=ws)
    torch.cuda.synchronize()
    ctx.check()
    m2 = cache.metrics_snapshot()
    assert m2["misses"] - m1["misses"] >= 1
    assert tier.stats()["failed"] == 1
    x = xs[2:3]
    h = None
    for l in range(N_LAYERS):
        ti = torch.from_numpy(idx[2, l][None].copy()).cuda()
        tw = torch.from_numpy(w[2, l][None].copy()).cuda()
        h = block_forward(ctx, layers[l], x, h, topk_idx=ti, topk_w=tw)
        if l + 1 < N_LAYERS:
            x = torch.from_numpy(O.rmsnorm_to_f16(h.cpu().numpy(), 1e-6).view(np.float16)).cuda()
    assert torch.equal(out, h)
    tier.close()
