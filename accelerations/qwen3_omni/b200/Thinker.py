"""B200 Thinker: the reference's Thinker program with every MoE layer's experts
on the sm_100a grouped tcgen05 kernels.

Same logical contract as accelerations/qwen3_omni/amd/Thinker.py (reference
ThinkerLogical; Inputs, Resources, Plans and Call unchanged, TensorForward
execution). The build is the reference's build_thinker
(implementations/qwen3_omni/amd/thinker_preparation.py:8-33; its
select_expert_kernels is a no-op off ROCm), after which
install_thinker_experts gives each MoE layer a ThinkerExpertsBackend: router
top-8 ids/weights -> counting-sort permutation -> gate/up GEMM with the SwiGLU
epilogue -> down GEMM with the routing-weight epilogue -> slot-ordered combine,
with the bf16 rounding points of thinker_moe.py:17-101; then
install_thinker_attention_linears makes the plain nn.Linear attention
projections (q/k/v/o_proj) and lm_head Q8_0 contractions (thinker_model.py:106-148,
the 48-layer stack's "linears in Q8_0"). No torch.compile: the program is
captured in CUDA graphs instead.

Requires the M* runtime (mstar); it is exercised through
python -m mstar_accelerators.testing --registry accelerations/qwen3_omni/b200.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch

from mstar.engine.resources.sampler.plan import SamplingPlan
from mstar.engine.resources.sequence_view import AttentionUse, SequenceUse
from mstar.engine.tensor_forward import CapturePolicy, CompilePolicy
from mstar.model.qwen3_omni.results import ThinkerResult
from mstar.model.qwen3_omni.thinker_logical import ThinkerLogical
from mstar_accelerators import Acceleration, Eq, Implementation, Range, TensorForwardExecution, When
from mstar_accelerators.backends.torch.tensor_forward import tensor_resource_requests
from mstar_accelerators_b200.conditions import SM100aAvailable
from mstar_accelerators_b200.moe import install_thinker_experts
from mstar_accelerators_b200.thinker import install_thinker_attention_linears


@dataclass(frozen=True)
class Inputs:
    input_ids: tuple[torch.Tensor | None, ...]
    media_embeds: tuple[torch.Tensor | None, ...]
    positions: tuple[torch.Tensor, ...]
    masks: tuple[torch.Tensor, ...]
    deepstack_0: tuple[torch.Tensor | None, ...]
    deepstack_1: tuple[torch.Tensor | None, ...]
    deepstack_2: tuple[torch.Tensor | None, ...]


class Resources:
    """Model-owned identities; physical views are chosen in implementation.resources."""
    thinker_kv = 'thinker_kv'
    thinker_attn = 'thinker_attn'
    thinker_pos = 'thinker_pos'
    thinker_sampler = 'thinker_sampler'


@dataclass(frozen=True)
class Plans:
    thinker_kv: dict[str, SequenceUse]
    thinker_attn: dict[str, AttentionUse]
    thinker_pos: dict[str, torch.Tensor]
    thinker_sampler: SamplingPlan


@dataclass(frozen=True)
class Call:
    graph_walk: Literal['prefill_audio', 'prefill_text', 'prefill_vision', 'thinker_decode']
    inputs: Inputs
    outputs: ThinkerResult
    plan_results: Plans
    row_walks: tuple[str, ...]


def build_thinker_b200(binding):
    from mstar_accelerators.implementations.qwen3_omni.amd.thinker_preparation import build_thinker
    program = build_thinker(binding)
    if install_thinker_experts(program) == 0:
        raise ValueError("no thinker MoE layer of the expected geometry was found")
    # attention-prologue projections and lm_head as Q8_0 contractions (plain nn.Linear only;
    # tensor-parallel linears keep their own path)
    install_thinker_attention_linears(program)
    return program


acceleration = Acceleration(
    reference=ThinkerLogical,
    when=When(Eq("node_name", "Thinker"), Eq("device_type", "cuda"), Eq("platform", "cuda"), SM100aAvailable(),
              Eq("dtype", torch.bfloat16), Eq("tp_size", 1), Eq("sp_size", 1), Range("batch_size", 1, 32)),
    implementation=Implementation(resources=tensor_resource_requests,
        execution=TensorForwardExecution(build=build_thinker_b200, bind_result=None,
            compile=CompilePolicy(enabled=False, fullgraph=False, dynamic=None, platform_overrides=False,
                                  fallback_to_eager=False),
            capture=CapturePolicy(enabled=True, required=False,
                compile=CompilePolicy(enabled=False, mode=None, fullgraph=False, dynamic=False,
                                      platform_overrides=False)),
            autocast_dtype=torch.bfloat16)))
