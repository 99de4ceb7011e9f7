"""qfmoe -- B200-native MoE-block hot path of QwenFieldfare.

Host-side package over libqf_moe.so (include/qf_moe.h).  The compute path is
hand-written sm_100a CUDA; there is no CPU fallback.
"""
from ._lib import QfError, lib  # noqa: F401
from .cache import ArenaLayer, ExpertCache, HostTier, plan_slots, stream_step  # noqa: F401
from .ep import ExpertParallel, exchange_handles  # noqa: F401
from .store import ExpertStore  # noqa: F401
from .moe import (  # noqa: F401
    DECODE_MAX_TOKENS, EXPERTS, HIDDEN, INTER, OFF, RECORD_BYTES, SHARED_EXPERT, TOPK,
    MoEContext, MoELayerWeights, StackPlan, block_forward, block_forward_prenorm, dispatch_plan, lm_head, router_logits,
    profile_begin, profile_end, router_topk, stack_forward, synth_hidden, synth_records,
    combine, grouped_ffn, routed_subset, shared_expert,
)
