"""Expert-parallel MoE block over NVLink (host side of qf_moe_block_forward_ep).

One process per GPU.  Rank r owns routed experts [r*256/world, (r+1)*256/world);
each rank routes its own tokens; rows move between GPUs by stores and loads on
CUDA-IPC-mapped peer memory inside the library's kernels.  torch.distributed is
used only to exchange the IPC handles and for host barriers.

The reference has no expert parallelism; the per-token math is the MoE step of
QwenQ4ActiveExpertStreamingRunner.forwardToken
(Sources/QwenFieldfareCore/Runtime/Generation/QwenQ4ActiveExpertStreamingRunner.swift:1169-1381).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import EP_HANDLE_BYTES, MoELayerDesc, QfError, check, lib
from .moe import EXPERTS, HIDDEN, TOPK, MoEContext, MoELayerWeights, _check_x, _ptr, _routing


def exchange_handles(handle: bytes, rank: int, world: int, group=None) -> bytes:
    """All ranks' IPC handles concatenated in rank order (a host all-gather)."""
    import torch.distributed as dist
    if len(handle) != EP_HANDLE_BYTES:
        raise ValueError("an EP handle is 64 bytes")
    if world == 1:
        return handle
    got = [None] * world
    dist.all_gather_object(got, (rank, handle), group=group)
    got.sort(key=lambda rh: rh[0])
    if [r for r, _ in got] != list(range(world)):
        raise RuntimeError("EP handle exchange: ranks are not 0..world-1")
    return b"".join(h for _, h in got)


class ExpertParallel:
    """Collective EP context: create on every rank with the same world and
    max_tokens, then call forward() the same number of times on every rank."""

    def __init__(self, ctx: MoEContext, rank: int, world: int, max_tokens: int, group=None):
        self.ctx = ctx
        self.rank, self.world, self.group = rank, world, group
        h = C.c_void_p()
        st = lib().qf_ep_create(ctx.h, rank, world, max_tokens, C.byref(h))
        if st != 0:
            raise QfError(st, lib().qf_last_error(ctx.h).decode())
        self.h = h
        self.max_tokens = max_tokens
        epr, rows, nbytes = C.c_int32(), C.c_int64(), C.c_uint64()
        check(lib().qf_ep_info(h, C.byref(epr), C.byref(rows), C.byref(nbytes)), ctx.h)
        self.experts_per_rank = epr.value
        self.receive_rows = rows.value
        self.region_bytes = nbytes.value
        self.first_expert = rank * self.experts_per_rank
        try:
            buf = (C.c_uint8 * EP_HANDLE_BYTES)()
            if world > 1:
                check(lib().qf_ep_ipc_handle(h, buf), ctx.h)
            allh = exchange_handles(bytes(buf), rank, world, group)
            arr = (C.c_uint8 * len(allh)).from_buffer_copy(allh)
            check(lib().qf_ep_connect(h, arr), ctx.h)
        except BaseException:
            lib().qf_ep_destroy(h)
            self.h = None
            raise
        self._barrier()

    def _barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def set_timeout_ms(self, ms: int):
        """Deadline of each bounded wait on the other ranks (default 2 s)."""
        check(lib().qf_ep_set_timeout_ms(self.h, ms), self.ctx.h)

    def set_down_at_home(self, enable: bool = True):
        """Owners return fp16 activation rows and each rank runs the down
        projection of its own tokens; the layer passed to forward() must then
        hold all 256 experts (every rank the same mode)."""
        check(lib().qf_ep_set_down_at_home(self.h, 1 if enable else 0), self.ctx.h)

    def local_layer(self, seed: int, layer: int) -> MoELayerWeights:
        """Seeded synthetic weights with this rank's experts in the bank."""
        return MoELayerWeights.synth(self.ctx, seed, layer, n_records=self.experts_per_rank,
                                     expert0=self.first_expert)

    def forward(self, layer: MoELayerWeights, x: torch.Tensor, residual: torch.Tensor | None = None,
                *, logit_bias=None, topk_idx=None, topk_w=None, out: torch.Tensor | None = None,
                return_routing: bool = False):
        _check_x(x)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, HIDDEN), dtype=torch.float32, device=self.ctx.device)
        idx = torch.empty((T, TOPK), dtype=torch.int32, device=self.ctx.device) if return_routing else None
        w = torch.empty((T, TOPK), dtype=torch.float32, device=self.ctx.device) if return_routing else None
        self.ctx._bind_stream()
        d = layer.desc()
        r = _routing(logit_bias, topk_idx, topk_w, None)
        check(lib().qf_moe_block_forward_ep(self.h, C.byref(d), T, _ptr(x), _ptr(residual), _ptr(out),
                                            C.byref(r) if r is not None else None, _ptr(idx),
                                            _ptr(w)), self.ctx.h)
        return (out, idx, w) if return_routing else out

    def close(self):
        """Collective: every rank's calls are complete before any region is freed."""
        if getattr(self, "h", None):
            torch.cuda.synchronize(self.ctx.device)
            self._barrier()
            lib().qf_ep_destroy(self.h)
            self.h = None


__all__ = ["ExpertParallel", "exchange_handles", "EXPERTS"]
