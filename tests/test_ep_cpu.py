"""Expert-parallel exchange on the CPU: two gloo ranks (world_size 2).

  - the product's IPC-handle exchange (qfmoe.ep.exchange_handles) hands every
    rank all handles in rank order;
  - the EP protocol (per-rank routing, counts all-gather, expert-major owner
    rows, owners evaluate their experts, results pulled back and combined in
    router order), modelled with the oracle's arithmetic in oracle/ep_sim.py,
    reproduces the single-process oracle block bit for bit, and the owner rows
    form a bijection.  The GPU kernels implement the same layout
    (tests/test_ep_gpu.py checks them against the single-GPU block).
No GPU is used."""
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEED, LAYER, T = 4, 2, 5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    for p in (os.path.join(ROOT, "qwen-fieldfare_b200"), os.path.join(ROOT, "oracle"), ROOT):
        sys.path.insert(0, p)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qfmoe.ep import exchange_handles
        import oracle as O
        import ep_sim
        mine = bytes([rank + 1]) * 64
        allh = exchange_handles(mine, rank, world)
        x16 = O.synth_hidden(SEED, 1000 + rank * T, T)
        res = np.random.default_rng(rank).standard_normal((T, O.HIDDEN)).astype(np.float32)
        out, idx, w, loc, qrows = ep_sim.ep_block(SEED, LAYER, x16, rank, world, residual=res)
        ref_layer = O.OracleLayer.synth(SEED, LAYER, experts=sorted(set(idx.reshape(-1).tolist())))
        ref = O.block(ref_layer, x16, residual=res, threads=2)
        q.put((rank, allh, bool(np.array_equal(out, ref["out"])), bool(np.array_equal(idx, ref["idx"])),
               loc.tolist(), qrows))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, allh, out_eq, idx_eq, loc, qrows = q.get(timeout=300)
        got[r] = (allh, out_eq, idx_eq, loc, qrows)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = b"".join(bytes([r + 1]) * 64 for r in range(world))
    for r in range(world):
        allh, out_eq, idx_eq, loc, qrows = got[r]
        assert allh == expect
        assert idx_eq and out_eq, r
    # every owner row is referenced by exactly one position of some rank
    for owner in range(world):
        rows = sorted(row for r in range(world) for d, row in got[r][3] if d == owner)
        assert rows == list(range(got[owner][4]))
