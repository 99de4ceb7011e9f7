"""CPU model of the expert-parallel exchange (test infrastructure only).

Restates, with the oracle's reference-order arithmetic, what the product's
expert-parallel block does across `world` ranks of a torch.distributed group:
  1. each rank routes its own tokens (router logits, top-8);
  2. positions sorted by (expert, token, k); per-expert counts all-gathered;
  3. each routed row goes to the owner of its expert (rank e // (256/world)) at
     row  sum_{owner's experts e' < e} total(e') + sum_{ranks s < me} count_s(e)
          + (rank of the row among my rows of e)
     (expert-major, then source rank, then (token, k)); on the wire a token
     row crosses once per owner: into the receive row of the token's lowest k
     with an expert there, which the owner's first-row map records at
     source rank * t_max + token; the token's other rows there carry that
     map index and the owner copies them from the first row (qf_ep.cu
     k_ep_dispatch, k_ep_expand);
  4. owners evaluate their experts on the received rows;
  5. each rank pulls its rows' results back and combines them in router order.
The per-token math is qfo_block's, so the outputs equal the single-process
oracle bit for bit.  Exchanges use all_gather_object (small test sizes).
"""
from __future__ import annotations

import numpy as np

try:
    from . import oracle as O  # package import
except ImportError:  # imported as a top-level module from the oracle directory
    import oracle as O


def dispatch_layout(board: np.ndarray, rank: int, world: int):
    """(base[256], q): the first owner row of this rank's rows of each expert,
    and the routed rows this rank receives, from the all-gathered counts
    board[world, 256]."""
    epr = O.EXPERTS // world
    total = board.sum(0)
    excl = np.cumsum(total) - total
    owner_first = (np.arange(O.EXPERTS) // epr) * epr
    base = excl - excl[owner_first] + board[:rank].sum(0)
    mine = slice(rank * epr, (rank + 1) * epr)
    return base.astype(np.int64), int(total[mine].sum())


def ep_block(seed: int, layer: int, x16: np.ndarray, rank: int, world: int, group=None,
             residual=None):
    """This rank's block output [T, 2048] (fp32) plus its routing (idx, w) and the
    (owner, row) of every position."""
    import torch.distributed as dist
    epr = O.EXPERTS // world
    T = x16.shape[0]
    L = O.OracleLayer.synth(seed, layer, experts=[])
    logits, coef = O.router(L, x16)
    idx, w = O.topk(logits)
    flat = idx.reshape(-1)
    perm = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=O.EXPERTS)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    boards = [None] * world
    dist.all_gather_object(boards, counts, group=group)
    board = np.stack(boards)
    base, q = dispatch_layout(board, rank, world)
    ts = [None] * world
    dist.all_gather_object(ts, T, group=group)
    t_max = max(ts)
    send_row = {d: [] for d in range(world)}  # (receive row, map index, token row): once per (token, owner)
    send_idx = {d: [] for d in range(world)}  # (receive row, map index): the other routed rows
    loc = np.zeros((T * O.TOPK, 2), np.int64)
    for j, pos in enumerate(perm):
        e = int(flat[pos])
        d = e // epr
        t, k = divmod(int(pos), O.TOPK)
        row = int(base[e] + j - offsets[e])
        trow = rank * t_max + t
        if all(int(flat[t * O.TOPK + kk]) // epr != d for kk in range(k)):
            send_row[d].append((row, trow, x16[t]))
        else:
            send_idx[d].append((row, trow))
        loc[pos] = (d, row)
    firsts = [None] * world
    idxs = [None] * world
    dist.all_gather_object(firsts, send_row, group=group)
    dist.all_gather_object(idxs, send_idx, group=group)
    recv = np.zeros((q, O.HIDDEN), np.uint16)
    placed = np.zeros(q, np.int64)
    first_row = {}
    for src in firsts:
        for row, trow, xr in src[rank]:
            if trow in first_row:
                raise AssertionError("a token row crossed twice to the same owner")
            first_row[trow] = row
            recv[row] = xr
            placed[row] += 1
    for src in idxs:
        for row, trow in src[rank]:
            recv[row] = recv[first_row[trow]]  # the expand step
            placed[row] += 1
    if not (placed == 1).all():
        raise AssertionError("owner rows are not a bijection")
    total = board.sum(0)
    y = np.zeros((q, O.HIDDEN), np.float32)
    row = 0
    for e in range(rank * epr, (rank + 1) * epr):
        if total[e] == 0:
            continue
        rec = O.synth_record(seed, layer, e)
        for _ in range(int(total[e])):
            y[row] = O.expert_ffn(rec, recv[row])
            row += 1
    results = [None] * world
    dist.all_gather_object(results, y, group=group)
    shared = O.synth_record(seed, layer, O.SHARED_EXPERT)
    out = np.empty((T, O.HIDDEN), np.float32)
    for t in range(T):
        y8 = np.stack([results[d][r] for d, r in loc[t * O.TOPK:(t + 1) * O.TOPK]])
        sh = O.expert_ffn(shared, x16[t])
        res = None if residual is None else residual[t]
        out[t] = O.combine(y8, w[t], sh, coef[t], res)
    return out, idx, w, loc, q
