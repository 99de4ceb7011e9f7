"""Python host mirror of the MoE step of QwenFieldfareCore over the C ABI.

Reference call sites this mirrors (tanishqpatil/qwen-fieldfare):
  - QwenQ4ActiveExpertStreamingRunner.forwardToken, MoE step
    (Sources/QwenFieldfareCore/Runtime/Generation/QwenQ4ActiveExpertStreamingRunner.swift:1169-1381)
  - QwenQ4ChatRunner.forwardToken resident MoE step (QwenQ4ChatRunner.swift:891-1000)
Device memory is torch-allocated; every compute call goes through libqf_moe.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import MoEDims, MoELayerDesc, QfError, RoutingDesc, check, lib

HIDDEN, EXPERTS, TOPK, INTER, GROUP = 2048, 256, 8, 512, 64
RECORD_BYTES = 1_769_472
SHARED_EXPERT = 256
DECODE_MAX_TOKENS = 64

# record layout (QwenQ4ExpertStoreBuilder.swift:47-56)
OFF = dict(gate_w=0, gate_s=524_288, gate_b=557_056, up_w=589_824, up_s=1_114_112,
           up_b=1_146_880, down_w=1_179_648, down_s=1_703_936, down_b=1_736_704)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class MoEContext:
    """One library handle bound to a CUDA device (replaces MetalContext)."""

    def __init__(self, device: int | torch.device = 0, scale_bf16: bool = False):
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("MoEContext needs a CUDA device; there is no CPU path")
        self.device = dev
        self.scale_bf16 = scale_bf16
        dims = MoEDims(HIDDEN, EXPERTS, TOPK, INTER, GROUP, 1 if scale_bf16 else 0)
        h = C.c_void_p()
        st = lib().qf_moe_create(C.byref(dims), dev.index or 0, C.byref(h))
        if st != 0:
            raise QfError(st, "qf_moe_create failed")
        self.h = h
        self._ws = {}

    def close(self):
        if getattr(self, "h", None):
            lib().qf_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _bind_stream(self):
        s = torch.cuda.current_stream(self.device)
        check(lib().qf_moe_set_stream(self.h, C.c_void_p(s.cuda_stream)), self.h)

    def check(self):
        """Synchronise and raise if a kernel flagged a violation."""
        self._bind_stream()
        check(lib().qf_moe_check(self.h), self.h)

    def workspace(self, T: int) -> torch.Tensor:
        n = C.c_size_t()
        check(lib().qf_moe_workspace_size(self.h, T, C.byref(n)), self.h)
        ws = self._ws.get(T)
        if ws is None or ws.numel() < n.value:
            ws = torch.empty(n.value, dtype=torch.uint8, device=self.device)
            self._ws[T] = ws
        return ws


@dataclass
class MoELayerWeights:
    """One layer's MoE weights in device memory, in the reference byte layout."""

    router_w: torch.Tensor  # uint8 [256*2048]
    router_s: torch.Tensor  # int16 bits [256*32]
    router_b: torch.Tensor
    coef_w: torch.Tensor    # uint8 [2048]
    coef_s: torch.Tensor    # int16 bits [32]
    coef_b: torch.Tensor
    shared: torch.Tensor    # uint8 [RECORD_BYTES]
    bank: torch.Tensor      # uint8 [n_records, RECORD_BYTES]

    def desc(self) -> MoELayerDesc:
        return MoELayerDesc(
            self.router_w.data_ptr(), self.router_s.data_ptr(), self.router_b.data_ptr(),
            self.coef_w.data_ptr(), self.coef_s.data_ptr(), self.coef_b.data_ptr(),
            self.shared.data_ptr(), self.bank.data_ptr(), self.bank.stride(0),
            self.bank.shape[0], 0)

    @classmethod
    def allocate(cls, device, n_records: int = EXPERTS):
        u8 = dict(dtype=torch.uint8, device=device)
        i16 = dict(dtype=torch.int16, device=device)
        return cls(torch.empty(EXPERTS * HIDDEN, **u8), torch.empty(EXPERTS * 32, **i16),
                   torch.empty(EXPERTS * 32, **i16), torch.empty(HIDDEN, **u8),
                   torch.empty(32, **i16), torch.empty(32, **i16),
                   torch.empty(RECORD_BYTES, **u8),
                   torch.empty((n_records, RECORD_BYTES), **u8))

    @classmethod
    def synth(cls, ctx: MoEContext, seed: int, layer: int, n_records: int = EXPERTS,
              bank: torch.Tensor | None = None, expert0: int = 0):
        """Seeded synthetic weights generated on the device (record i holds expert
        expert0 + i; an expert-parallel rank passes its first expert)."""
        w = cls.allocate(ctx.device, 0 if bank is not None else n_records)
        if bank is not None:
            w.bank = bank
        ctx._bind_stream()
        L = lib()
        check(L.qf_synth_router(ctx.h, seed, layer, _ptr(w.router_w), _ptr(w.router_s),
                                _ptr(w.router_b)), ctx.h)
        check(L.qf_synth_coef(ctx.h, seed, layer, _ptr(w.coef_w), _ptr(w.coef_s),
                              _ptr(w.coef_b)), ctx.h)
        check(L.qf_synth_records(ctx.h, seed, layer, SHARED_EXPERT, 1, _ptr(w.shared),
                                 RECORD_BYTES), ctx.h)
        if w.bank.shape[0] > 0:
            check(L.qf_synth_records(ctx.h, seed, layer, expert0,
                                     min(w.bank.shape[0], EXPERTS - expert0),
                                     _ptr(w.bank), w.bank.stride(0)), ctx.h)
        return w


def synth_records(ctx: MoEContext, seed: int, layer: int, expert0: int, count: int,
                  dst: torch.Tensor) -> None:
    """Generate `count` expert records into rows of dst ([count, stride] uint8)."""
    ctx._bind_stream()
    check(lib().qf_synth_records(ctx.h, seed, layer, expert0, count, _ptr(dst), dst.stride(0)),
          ctx.h)


def synth_hidden(seed: int, tok0: int, T: int) -> torch.Tensor:
    """Seeded fp16 hidden states (host tensor [T, 2048]): N(0,1), RMS-normalised."""
    x = torch.empty((T, HIDDEN), dtype=torch.float16)
    lib().qf_synth_hidden_host(seed, tok0, T, C.c_void_p(x.data_ptr()))
    return x


def _routing(bias=None, idx=None, w=None, record_of_pos=None):
    if bias is None and idx is None and record_of_pos is None:
        return None
    return RoutingDesc(None if bias is None else bias.data_ptr(),
                       None if idx is None else idx.data_ptr(),
                       None if w is None else w.data_ptr(),
                       None if record_of_pos is None else record_of_pos.data_ptr())


def _check_x(x: torch.Tensor):
    if x.dtype != torch.float16 or x.dim() != 2 or x.shape[1] != HIDDEN or not x.is_contiguous():
        raise ValueError("x must be a contiguous float16 tensor [T, 2048]")


def router_logits(ctx: MoEContext, layer: MoELayerWeights, x: torch.Tensor, want_coef=True):
    """qwen_router_q8_logits_simd_f32 (+ shared-gate coefficient): logits [T,256], coef [T]."""
    _check_x(x)
    T = x.shape[0]
    logits = torch.empty((T, EXPERTS), dtype=torch.float32, device=ctx.device)
    coef = torch.empty(T, dtype=torch.float32, device=ctx.device) if want_coef else None
    ctx._bind_stream()
    d = layer.desc()
    check(lib().qf_router_logits_q8(ctx.h, C.byref(d), T, _ptr(x), _ptr(logits), _ptr(coef)),
          ctx.h)
    return logits, coef


def router_topk(ctx: MoEContext, logits: torch.Tensor, bias: torch.Tensor | None = None):
    """qwen_router_top8_logits_f32: (idx int32 [T,8], w fp32 [T,8])."""
    T = logits.shape[0]
    idx = torch.empty((T, TOPK), dtype=torch.int32, device=ctx.device)
    w = torch.empty((T, TOPK), dtype=torch.float32, device=ctx.device)
    ctx._bind_stream()
    check(lib().qf_router_topk(ctx.h, _ptr(logits), _ptr(bias), T, _ptr(idx), _ptr(w)), ctx.h)
    return idx, w


def lm_head(ctx: MoEContext, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
            x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Q4 LM-head logits (qwen_gemv_q4_affine_simd_f32, reference order): w uint8
    [rows, 1024], scales / biases int16 bits [rows, 32] in the context's scale
    dtype, x fp32 [T, 2048] -> logits fp32 [T, rows]."""
    rows = w.shape[0]
    if x.dim() == 1:
        x = x[None]
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, rows), dtype=torch.float32, device=ctx.device)
    ctx._bind_stream()
    check(lib().qf_lm_head_q4(ctx.h, _ptr(w), _ptr(scales), _ptr(biases), rows, T, _ptr(x), _ptr(out)),
          ctx.h)
    return out


def dispatch_plan(ctx: MoEContext, idx: torch.Tensor):
    """Stable dispatch plan: counts [256], offsets [257], perm [T*8] (by expert, token, k)."""
    T = idx.shape[0]
    n = C.c_size_t()
    check(lib().qf_moe_dispatch_workspace_size(ctx.h, T, C.byref(n)), ctx.h)
    ws = torch.empty(max(n.value, 16), dtype=torch.uint8, device=ctx.device)
    counts = torch.empty(EXPERTS, dtype=torch.int32, device=ctx.device)
    offsets = torch.empty(EXPERTS + 1, dtype=torch.int32, device=ctx.device)
    perm = torch.empty(T * TOPK, dtype=torch.int32, device=ctx.device)
    ctx._bind_stream()
    check(lib().qf_moe_dispatch_plan(ctx.h, _ptr(idx), T, _ptr(counts), _ptr(offsets),
                                     _ptr(perm), _ptr(ws), ws.numel()), ctx.h)
    return counts, offsets, perm


def block_forward(ctx: MoEContext, layer: MoELayerWeights, x: torch.Tensor,
                  residual: torch.Tensor | None = None, *, logit_bias=None, topk_idx=None,
                  topk_w=None, record_of_pos=None, out: torch.Tensor | None = None,
                  return_routing: bool = False):
    """One MoE block: out = residual + shared(x) + sum_k w_k expert_k(x)."""
    _check_x(x)
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device=ctx.device)
    idx = torch.empty((T, TOPK), dtype=torch.int32, device=ctx.device) if return_routing else None
    w = torch.empty((T, TOPK), dtype=torch.float32, device=ctx.device) if return_routing else None
    ws = ctx.workspace(T)
    ctx._bind_stream()
    d = layer.desc()
    r = _routing(logit_bias, topk_idx, topk_w, record_of_pos)
    check(lib().qf_moe_block_forward(ctx.h, C.byref(d), T, _ptr(x), _ptr(residual), _ptr(out),
                                     C.byref(r) if r is not None else None, _ptr(idx), _ptr(w),
                                     _ptr(ws), ws.numel()), ctx.h)
    return (out, idx, w) if return_routing else out


def routed_subset(ctx: MoEContext, layer: MoELayerWeights, x: torch.Tensor, slot_of_pos: torch.Tensor,
                  w: torch.Tensor, positions, out: torch.Tensor | None = None,
                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts of a subset of one token's top-8 positions (the hit or the
    miss set of the streaming runner): fp32 [1, 2048] = sum over the listed
    positions, in list order, of w[p] * expert_p(x) (qf_moe_routed_subset).
    layer.bank is the slot arena; slot_of_pos int32 [8] and w fp32 [8] on the
    device; positions: a list of distinct ints in [0, 8)."""
    _check_x(x)
    if x.shape[0] != 1:
        raise ValueError("a subset is one token's")
    pos = torch.tensor(list(positions) + [0] * (TOPK - len(positions)), dtype=torch.int32,
                       device=ctx.device)
    if out is None:
        out = torch.empty((1, HIDDEN), dtype=torch.float32, device=ctx.device)
    ws = workspace if workspace is not None else ctx.workspace(1)
    ctx._bind_stream()
    d = layer.desc()
    check(lib().qf_moe_routed_subset(ctx.h, C.byref(d), _ptr(x), _ptr(slot_of_pos), _ptr(w), _ptr(pos),
                                     len(positions), _ptr(out), _ptr(ws), ws.numel()), ctx.h)
    return out


def shared_expert(ctx: MoEContext, layer: MoELayerWeights, x: torch.Tensor, coef: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """sigmoid(coef[t]) * shared_expert(x_t) for T <= 64 tokens (qf_shared_expert)."""
    _check_x(x)
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device=ctx.device)
    ws = ctx.workspace(T)
    ctx._bind_stream()
    d = layer.desc()
    check(lib().qf_shared_expert(ctx.h, C.byref(d), T, _ptr(x), _ptr(coef), _ptr(out), _ptr(ws),
                                 ws.numel()), ctx.h)
    return out


def combine(ctx: MoEContext, shared_out: torch.Tensor, residual: torch.Tensor | None = None,
            hit: torch.Tensor | None = None, miss: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """((residual + shared_out) + hit) + miss, a None term being 0 (qf_moe_combine)."""
    T = shared_out.shape[0]
    if out is None:
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device=ctx.device)
    ctx._bind_stream()
    check(lib().qf_moe_combine(ctx.h, T, _ptr(residual), _ptr(shared_out), _ptr(hit), _ptr(miss),
                               _ptr(out)), ctx.h)
    return out


def grouped_ffn(ctx: MoEContext, layer: MoELayerWeights, x: torch.Tensor, idx: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Unweighted routed expert outputs of every position, fp32 [T * 8, 2048]:
    row t * 8 + k = expert idx[t, k] applied to x_t (qf_moe_grouped_ffn)."""
    _check_x(x)
    T = x.shape[0]
    if out is None:
        out = torch.empty((T * TOPK, HIDDEN), dtype=torch.float32, device=ctx.device)
    n = C.c_size_t()
    check(lib().qf_moe_grouped_ffn_workspace_size(ctx.h, T, C.byref(n)), ctx.h)
    ws = torch.empty(n.value, dtype=torch.uint8, device=ctx.device)
    ctx._bind_stream()
    d = layer.desc()
    check(lib().qf_moe_grouped_ffn(ctx.h, C.byref(d), T, _ptr(x), _ptr(idx), _ptr(out), _ptr(ws),
                                   ws.numel()), ctx.h)
    return out


def block_forward_prenorm(ctx: MoEContext, layer: MoELayerWeights, hidden: torch.Tensor,
                          norm_w: torch.Tensor, eps: float = 1e-6, *, out: torch.Tensor | None = None,
                          return_routing: bool = False):
    """The block from the residual stream: x = fp16(RMSNorm(hidden) * norm_w) in the
    reference kernel's order, then block_forward(x, residual=hidden)."""
    if hidden.dtype != torch.float32 or hidden.dim() != 2 or hidden.shape[1] != HIDDEN:
        raise ValueError("hidden must be float32 [T, 2048]")
    T = hidden.shape[0]
    if out is None:
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device=ctx.device)
    idx = torch.empty((T, TOPK), dtype=torch.int32, device=ctx.device) if return_routing else None
    w = torch.empty((T, TOPK), dtype=torch.float32, device=ctx.device) if return_routing else None
    n = C.c_size_t()
    check(lib().qf_moe_workspace_size(ctx.h, T, C.byref(n)), ctx.h)
    need = (n.value + 255) // 256 * 256 + T * HIDDEN * 2
    ws = ctx._ws.get(("prenorm", T))
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=ctx.device)
        ctx._ws[("prenorm", T)] = ws
    ctx._bind_stream()
    d = layer.desc()
    check(lib().qf_moe_block_forward_prenorm(ctx.h, C.byref(d), T, _ptr(hidden), _ptr(norm_w), eps,
                                             _ptr(out), None, _ptr(idx), _ptr(w), _ptr(ws), ws.numel()),
          ctx.h)
    return (out, idx, w) if return_routing else out


class StackPlan:
    """Host array of layer descriptors for qf_moe_stack_forward."""

    def __init__(self, layers):
        self.layers = list(layers)
        self.arr = (MoELayerDesc * len(self.layers))(*[l.desc() for l in self.layers])


def stack_forward(ctx: MoEContext, plan: StackPlan, x: torch.Tensor,
                  residual: torch.Tensor | None = None, eps: float = 1e-6,
                  out: torch.Tensor | None = None, return_routing: bool = False,
                  workspace: torch.Tensor | None = None):
    """n stacked blocks: h_{l+1} = out_l, x_{l+1} = fp16(RMSNorm(out_l))."""
    _check_x(x)
    T = x.shape[0]
    n = len(plan.layers)
    if out is None:
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device=ctx.device)
    idx = torch.empty((n, T, TOPK), dtype=torch.int32, device=ctx.device) if return_routing else None
    w = torch.empty((n, T, TOPK), dtype=torch.float32, device=ctx.device) if return_routing else None
    ws = workspace if workspace is not None else ctx.workspace(T)
    ctx._bind_stream()
    check(lib().qf_moe_stack_forward(ctx.h, plan.arr, n, T, _ptr(x), _ptr(residual), _ptr(out),
                                     eps, _ptr(idx), _ptr(w), _ptr(ws), ws.numel()), ctx.h)
    return (out, idx, w) if return_routing else out


KERNEL_IDS = {"router": 0, "topk": 1, "gate_up": 2, "down": 3, "combine": 4, "fused": 5,
              "dispatch": 6}


def profile_begin(ctx: MoEContext, kernel: str, max_launches: int = 4096) -> None:
    """Record CUDA events around every launch of one block kernel (bench timing)."""
    check(lib().qf_moe_profile_begin(ctx.h, KERNEL_IDS[kernel], max_launches), ctx.h)


def profile_end(ctx: MoEContext):
    """(total_ms, launches) of the launches recorded since profile_begin."""
    ms = C.c_float()
    n = C.c_int32()
    check(lib().qf_moe_profile_end(ctx.h, C.byref(ms), C.byref(n)), ctx.h)
    return ms.value, n.value
