"""The allocation-free block entry point, qf_moe_block_forward_static.

It serves callers that cannot call cudaMalloc when they run the MoE block (an
engine that owns all device memory through its own arena, a language binding
without a device allocator, a step that must stay off the allocator): its
scratch lives in a 1 MiB device array inside the library.  These tests call it
through the C ABI and check it against qf_moe_block_forward (the entry point
that takes a caller-provided workspace) and against the CPU oracle, on two
calls in a row (the shared array keeps the previous call's contents), with
fp16 and bf16 scales; that free device memory does not change across calls;
and that every descriptor qf_moe_block_forward rejects is rejected here too,
with QF_ERR_ARG and nothing written.  Collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def free_bytes():
    f, _ = torch.cuda.mem_get_info()  # cudaMemGetInfo: free device memory
    return f


def call_static(scale_dtype, desc, T, x, res, out, idx, w):
    from qfmoe._lib import lib
    stream = torch.cuda.current_stream()
    return lib().qf_moe_block_forward_static(
        scale_dtype, C.byref(desc), T, C.c_void_p(x.data_ptr()),
        None if res is None else C.c_void_p(res.data_ptr()), C.c_void_p(out.data_ptr()),
        None if idx is None else C.c_void_p(idx.data_ptr()),
        None if w is None else C.c_void_p(w.data_ptr()), C.c_void_p(stream.cuda_stream))


@pytest.mark.parametrize("bf16", [False, True], ids=["f16_scales", "bf16_scales"])
def test_static_entry_matches_workspace_entry_and_oracle_twice(bf16):
    import qfmoe as Q

    seed, lyr = 4, 3
    ctx = Q.MoEContext(0, scale_bf16=bf16)
    layer = Q.MoELayerWeights.synth(ctx, seed=seed, layer=lyr)
    olayer = O.OracleLayer.synth(seed, lyr, bf16=bf16)
    desc = layer.desc()
    for call, (T, tok0) in enumerate([(8, 0), (3, 500)]):
        x = Q.synth_hidden(seed, tok0, T)
        res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(call))
        ref, ridx, rw = Q.block_forward(ctx, layer, x.cuda(), res.cuda(), return_routing=True)
        xo = x.numpy().view(np.uint16)
        oref = O.block(olayer, xo, residual=res.numpy(), threads=8)
        xd, resd = x.cuda(), res.cuda()
        out = torch.full((T, 2048), float("nan"), device="cuda")
        idx = torch.full((T, 8), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros((T, 8), device="cuda")
        torch.cuda.synchronize()
        before = free_bytes() if call == 1 else None
        assert call_static(1 if bf16 else 0, desc, T, xd, resd, out, idx, w) == 0
        torch.cuda.synchronize()
        if before is not None:
            assert free_bytes() == before  # the second call allocates nothing
        assert torch.equal(idx, ridx)
        assert np.array_equal(idx.cpu().numpy(), oref["idx"])
        assert max_rel(w.cpu().numpy(), rw.cpu().numpy()) < 1e-6
        assert max_rel(w.cpu().numpy(), oref["w"]) < 1e-5
        got = out.cpu().numpy()
        assert max_rel(got, ref.cpu().numpy()) < TOL
        err = max_rel(got, oref["out"])
        assert err < TOL, (call, err)


SPOILERS = [
    ("coef_w + 8", lambda d: setattr(d, "coef_w", d.coef_w + 8)),
    ("router_w + 4", lambda d: setattr(d, "router_w", d.router_w + 4)),
    ("coef_s + 1", lambda d: setattr(d, "coef_s", d.coef_s + 1)),
    ("expert_bank + 16", lambda d: setattr(d, "expert_bank", d.expert_bank + 16)),
    ("record_stride + 16", lambda d: setattr(d, "record_stride", d.record_stride + 16)),
    ("bank_records 0", lambda d: setattr(d, "bank_records", 0)),
]


def test_static_entry_rejects_what_the_workspace_entry_rejects():
    import qfmoe as Q
    from qfmoe._lib import MoELayerDesc, lib

    ctx = Q.MoEContext(0)
    layer = Q.MoELayerWeights.synth(ctx, seed=4, layer=3)
    T = 2
    x = Q.synth_hidden(4, 0, T).cuda()
    ws_bytes = C.c_size_t()
    assert lib().qf_moe_workspace_size(ctx.h, T, C.byref(ws_bytes)) == 0
    ws = torch.empty(ws_bytes.value + 256, dtype=torch.uint8, device="cuda")
    for name, spoil in SPOILERS:
        d = MoELayerDesc.from_buffer_copy(layer.desc())
        spoil(d)
        out = torch.full((T, 2048), float("nan"), device="cuda")
        torch.cuda.synchronize()
        assert call_static(0, d, T, x, None, out, None, None) == -1, name  # QF_ERR_ARG
        assert lib().qf_moe_block_forward(
            ctx.h, C.byref(d), T, C.c_void_p(x.data_ptr()), None, C.c_void_p(out.data_ptr()),
            None, None, None, C.c_void_p(ws.data_ptr()), ws_bytes.value) == -1, name
        torch.cuda.synchronize()
        assert torch.isnan(out).all(), name  # nothing was launched
    # the good descriptor still runs after the rejected calls
    out = torch.full((T, 2048), float("nan"), device="cuda")
    assert call_static(0, layer.desc(), T, x, None, out, None, None) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_static_entry_rejects_more_than_eight_tokens():
    import qfmoe as Q

    ctx = Q.MoEContext(0)
    layer = Q.MoELayerWeights.synth(ctx, seed=4, layer=3, n_records=256)
    x = Q.synth_hidden(4, 0, 9).cuda()
    out = torch.full((9, 2048), float("nan"), device="cuda")
    assert call_static(0, layer.desc(), 9, x, None, out, None, None) == -1  # QF_ERR_ARG
    torch.cuda.synchronize()
    assert torch.isnan(out).all()
