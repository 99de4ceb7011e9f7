"""Expert-parallel block on the GPU against the single-GPU block.

world 1 (one GPU) runs the whole EP path -- count board, dispatch by stores
into the exported region, grouped GEMMs over the received rows, pull combine --
against itself, and must equal qf_moe_block_forward bit for bit.  world 2 (two
GPUs, one process each, skipped with fewer GPUs) moves rows over NVLink; every
rank's output must equal the single-GPU block on the same tokens bit for bit."""
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEED, LAYER = 6, 1
TOL = 2e-3


def zipf_bias(s=1.1):
    rng = np.random.default_rng(3)
    order = rng.permutation(256)
    p = 1.0 / np.arange(1, 257) ** s
    b = np.empty(256, np.float32)
    b[order] = np.log(p / p.max())
    return b


def max_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="module")
def full_layer(ctx):
    from qfmoe import MoELayerWeights
    return MoELayerWeights.synth(ctx, SEED, LAYER)


def test_ep_world1_equals_block(ctx, full_layer):
    from qfmoe import ExpertParallel, block_forward, synth_hidden
    ep = ExpertParallel(ctx, 0, 1, max_tokens=512)
    bias = torch.from_numpy(zipf_bias()).cuda()
    for i, T in enumerate((300, 512, 97, 300)):
        x = synth_hidden(SEED, 1000 * i, T).cuda()
        res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(i)).cuda()
        out, idx, w = ep.forward(full_layer, x, res, logit_bias=bias, return_routing=True)
        ref, ridx, rw = block_forward(ctx, full_layer, x, res, logit_bias=bias, return_routing=True)
        ctx.check()
        assert torch.equal(idx, ridx) and torch.equal(w, rw)
        assert torch.equal(out, ref), (T, (out - ref).abs().max().item())
    ep.close()


def test_ep_world1_down_at_home_equals_block(ctx, full_layer):
    """Down-at-home mode: the owner returns activation rows and the home rank
    runs the down projection with all 256 experts; same outputs bit for bit.
    A bank with fewer than 256 experts is refused in this mode."""
    from qfmoe import ExpertParallel, MoELayerWeights, QfError, block_forward, synth_hidden
    ep = ExpertParallel(ctx, 0, 1, max_tokens=512)
    ep.set_down_at_home(True)
    bias = torch.from_numpy(zipf_bias()).cuda()
    for i, T in enumerate((300, 512, 97)):
        x = synth_hidden(SEED, 3000 + 1000 * i, T).cuda()
        res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(50 + i)).cuda()
        out, idx, w = ep.forward(full_layer, x, res, logit_bias=bias if i else None, return_routing=True)
        ref, ridx, rw = block_forward(ctx, full_layer, x, res, logit_bias=bias if i else None, return_routing=True)
        ctx.check()
        assert torch.equal(idx, ridx)
        assert torch.equal(out, ref), (T, (out - ref).abs().max().item())
    small = MoELayerWeights.synth(ctx, SEED, LAYER, n_records=128)
    with pytest.raises(QfError):
        ep.forward(small, synth_hidden(SEED, 0, 8).cuda())
    ep.set_down_at_home(False)
    # (T > 64: block_forward takes the prefill path, whose router the EP block uses)
    x = synth_hidden(SEED, 9000, 128).cuda()
    assert torch.equal(ep.forward(full_layer, x), block_forward(ctx, full_layer, x))
    ep.close()


def test_ep_world1_small_batch_vs_oracle(ctx, full_layer):
    from qfmoe import ExpertParallel, synth_hidden
    ep = ExpertParallel(ctx, 0, 1, max_tokens=16)
    x = synth_hidden(SEED, 77, 5)
    out, idx, _ = ep.forward(full_layer, x.cuda(), return_routing=True)
    ctx.check()
    OL = O.OracleLayer.synth(SEED, LAYER, experts=sorted(set(idx.cpu().numpy().reshape(-1).tolist())))
    ref = O.block(OL, x.numpy().view(np.uint16), threads=8)
    assert np.array_equal(idx.cpu().numpy(), ref["idx"])
    assert max_rel(out.cpu().numpy(), ref["out"]) < TOL
    ep.close()


def test_ep_supplied_routing_and_argument_errors(ctx, full_layer):
    from qfmoe import ExpertParallel, QfError, block_forward, synth_hidden
    ep = ExpertParallel(ctx, 0, 1, max_tokens=128)
    T = 128
    rng = np.random.default_rng(2)
    idx = torch.from_numpy(np.stack([rng.choice(256, 8, replace=False) for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.random((T, 8)).astype(np.float32)).cuda()
    x = synth_hidden(SEED, 5000, T).cuda()
    out = ep.forward(full_layer, x, topk_idx=idx, topk_w=w)
    ref = block_forward(ctx, full_layer, x, topk_idx=idx, topk_w=w)
    ctx.check()
    assert torch.equal(out, ref)
    with pytest.raises(QfError):  # more tokens than max_tokens
        ep.forward(full_layer, synth_hidden(SEED, 0, 129).cuda())
    ep.close()
    for rank, world in ((0, 3), (2, 2), (0, 16)):  # world must divide 256 and be <= 8
        with pytest.raises(QfError):
            ExpertParallel(ctx, rank, world, max_tokens=16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    for p in (os.path.join(ROOT, "qwen-fieldfare_b200"), os.path.join(ROOT, "oracle"), ROOT):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        import qfmoe as Q
        ctx = Q.MoEContext(rank)
        # ranks created with different max_tokens refuse to connect
        try:
            Q.ExpertParallel(ctx, rank, world, max_tokens=256 + 128 * rank)
            mismatch_refused = False
        except Q.QfError:
            mismatch_refused = True
        dist.barrier()
        T = 384
        ep = Q.ExpertParallel(ctx, rank, world, max_tokens=T)
        local = ep.local_layer(SEED, LAYER)
        full = Q.MoELayerWeights.synth(ctx, SEED, LAYER)
        bias = torch.from_numpy(zipf_bias()).cuda()
        equal = []
        for step in range(6):
            # steps 4, 5: down-at-home mode (all 256 experts on each rank)
            if step == 4:
                ep.set_down_at_home(True)
            x = Q.synth_hidden(SEED, 10000 * step + rank * T, T).cuda()
            res = torch.randn((T, 2048), generator=torch.Generator().manual_seed(100 * step + rank)).cuda()
            out = ep.forward(local if step < 4 else full, x, res, logit_bias=bias if step % 2 else None)
            ref = Q.block_forward(ctx, full, x, res, logit_bias=bias if step % 2 else None)
            ctx.check()
            equal.append(bool(torch.equal(out, ref)))
        ep.close()
        q.put((rank, mismatch_refused, equal, None))
    except Exception as exc:  # reported to the parent
        q.put((rank, None, None, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ep_two_gpus_equals_single_gpu_block():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, refused, equal, err = q.get(timeout=600)
        got[r] = (refused, equal, err)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        refused, equal, err = got[r]
        assert err is None, err
        assert refused, "mismatched max_tokens must be refused"
        assert all(equal), (r, equal)


def _timeout_worker(rank, world, port, q, dev, down_at_home=False):
    """Rank 1 creates and connects, then leaves the group: it never calls
    forward, but keeps its exported region alive (rank 0 stores into it) until
    rank 0 has finished.  Rank 0 calls forward with a 50 ms deadline."""
    for p in (os.path.join(ROOT, "qwen-fieldfare_b200"), os.path.join(ROOT, "oracle"), ROOT):
        sys.path.insert(0, p)
    import datetime
    import time
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(dev)
        import qfmoe as Q
        from qfmoe._lib import lib
        ctx = Q.MoEContext(dev)
        # above 64 tokens the single-GPU block takes the prefill router, as EP
        # does, so the two outputs compare bit for bit
        T = 96
        ep = Q.ExpertParallel(ctx, rank, world, max_tokens=T)
        if rank == 1:
            dist.barrier()  # rank 0 is done with our region
            lib().qf_ep_destroy(ep.h)
            ep.h = None
            q.put((rank, None, None))
            return
        ep.set_timeout_ms(50)
        if down_at_home:
            ep.set_down_at_home(True)
            layer = Q.MoELayerWeights.synth(ctx, SEED, LAYER)
        else:
            layer = ep.local_layer(SEED, LAYER)
        x = Q.synth_hidden(SEED, 0, T).cuda()
        t0 = time.time()
        ep.forward(layer, x)
        torch.cuda.synchronize()
        elapsed = time.time() - t0
        try:
            ctx.check()
            status = "ok"
        except Q.QfError as e:
            status = str(e)
        ctx.check()  # the status word was cleared
        lib().qf_ep_destroy(ep.h)  # the group is broken: no collective close
        ep.h = None
        # the handle stays usable: a world-1 EP call and a plain block
        full = Q.MoELayerWeights.synth(ctx, SEED, LAYER)
        ep1 = Q.ExpertParallel(ctx, 0, 1, max_tokens=T)
        out1 = ep1.forward(full, x)
        ref = Q.block_forward(ctx, full, x)
        ctx.check()
        ep1.close()
        dist.barrier()  # let rank 1 free its region
        q.put((rank, (status, elapsed, bool(torch.equal(out1, ref))), None))
    except Exception as exc:  # reported to the parent
        try:
            dist.barrier()
        except Exception:
            pass
        q.put((rank, None, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("down_at_home", [False, True], ids=["sharded", "down_at_home"])
def test_ep_missing_rank_times_out_and_the_handle_recovers(down_at_home):
    """A rank that never arrives: rank 0's bounded waits expire after the 50 ms
    deadline, qf_moe_check reports QF_ERR_TIMEOUT, the call's GEMMs do no work,
    and a following world-1 call on the same handle equals the single-GPU block.
    Only rank 0 launches kernels; with two or more GPUs the ranks sit on
    different GPUs, with one both processes share it (rank 1 only holds its
    exported region)."""
    world = 2
    two = torch.cuda.device_count() >= 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, world, port, q, r if two else 0, down_at_home))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, res, err = q.get(timeout=600)
        got[r] = (res, err)
    for p in procs:
        p.join(timeout=120)
    assert got[1][1] is None, got[1][1]
    res, err = got[0]
    assert err is None, err
    status, elapsed, equal = res
    assert "QF_ERR_TIMEOUT" in status, status
    assert elapsed < 5.0, elapsed  # 50 ms deadlines, not the 2 s default
    assert equal
