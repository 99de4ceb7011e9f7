"""The allocation-free block entry point, qf_moe_block_forward_static.

It serves callers that cannot call cudaMalloc when they run the MoE block (an
engine that owns all device memory through its own arena, a language binding
without a device allocator, a step that must stay off the allocator): its
scratch lives in a 1 MiB device array inside the library.  This test calls it
through the C ABI and checks it against qf_moe_block_forward, the entry point
that takes a caller-provided workspace, on two calls in a row (the shared
array keeps the previous call's contents), and that free device memory does
not change across calls.  Collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL = 2e-3


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def free_bytes():
    f, _ = torch.cuda.mem_get_info()  # cudaMemGetInfo: free device memory
    return f


def test_static_entry_matches_workspace_entry_twice():
    import qfmoe as Q
    from qfmoe._lib import lib

    ctx = Q.MoEContext(0)
    layer = Q.MoELayerWeights.synth(ctx, seed=4, layer=3)
    desc = layer.desc()
    stream = torch.cuda.current_stream()
    results = []
    for call, (T, tok0) in enumerate([(8, 0), (3, 500)]):
        x = Q.synth_hidden(4, tok0, T).cuda()
        res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(call)).cuda()
        ref, ridx, rw = Q.block_forward(ctx, layer, x, res, return_routing=True)
        out = torch.full((T, 2048), float("nan"), device="cuda")
        idx = torch.full((T, 8), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros((T, 8), device="cuda")
        torch.cuda.synchronize()
        before = free_bytes() if call == 1 else None
        st = lib().qf_moe_block_forward_static(
            0, C.byref(desc), T, C.c_void_p(x.data_ptr()), C.c_void_p(res.data_ptr()),
            C.c_void_p(out.data_ptr()), C.c_void_p(idx.data_ptr()), C.c_void_p(w.data_ptr()),
            C.c_void_p(stream.cuda_stream))
        assert st == 0
        torch.cuda.synchronize()
        if before is not None:
            assert free_bytes() == before  # the second call allocates nothing
        assert torch.equal(idx, ridx)
        assert max_rel(w.cpu().numpy(), rw.cpu().numpy()) < 1e-6
        err = max_rel(out.cpu().numpy(), ref.cpu().numpy())
        assert err < TOL, err
        results.append(err)
    assert len(results) == 2


def test_static_entry_rejects_more_than_eight_tokens():
    import qfmoe as Q
    from qfmoe._lib import lib

    ctx = Q.MoEContext(0)
    layer = Q.MoELayerWeights.synth(ctx, seed=4, layer=3, n_records=256)
    desc = layer.desc()
    x = Q.synth_hidden(4, 0, 9).cuda()
    out = torch.empty((9, 2048), device="cuda")
    st = lib().qf_moe_block_forward_static(0, C.byref(desc), 9, C.c_void_p(x.data_ptr()), None,
                                           C.c_void_p(out.data_ptr()), None, None, None)
    assert st == -1  # QF_ERR_ARG
