"""B200 Whisper audio encoder: the stock-Q8 encoder graph on sm_100a kernels.

Same logical contract as accelerations/whisper/pi_cpu/audio_encoder.py
(reference WhisperEncoderSubmodule, prefill walk, audio_features per row
(80, 3000) fp32 -> encoder_states per row (1500, 384) fp32, written into the
call's owned outputs) gated by the sm_100a device Condition instead of
CPUQ8EncoderAvailable. All rows of one call are encoded together (the
reference admits batch_size 1 only). The Q8_0 GEMMs, staging, LayerNorm and
fused epilogues are this package's kernels; the attention between them is
torch's scaled-dot-product attention over the zero-padded fp16 K/V planes.

Requires the M* runtime (mstar); it is exercised through
python -m mstar_accelerators.testing --registry accelerations/whisper/b200.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch

from mstar.model.whisper.results import EncoderResult
from mstar.model.whisper.submodules import WhisperEncoderSubmodule
from mstar_accelerators import Acceleration, Eq, Implementation, PreparedImplementation, Range, When
from mstar_accelerators.backends.weights import prepare_weights
from mstar_accelerators.compiler import bind_default_call, default_resource_requests
from mstar_accelerators_b200.conditions import SM100aAvailable
from mstar_accelerators_b200.encoder import TINY, WhisperEncoderB200
from mstar_accelerators_b200.programs import DeviceProgram, prepare_device_programs

MAX_ROWS = 16


@dataclass(frozen=True)
class Inputs:
    audio_features: tuple[torch.Tensor, ...]  # per-row shape (80, 3000)


class Resources:
    """Model-owned identities; physical views are chosen in implementation.resources."""


@dataclass(frozen=True)
class Plans:
    pass


@dataclass(frozen=True)
class Call:
    graph_walk: Literal['prefill']
    inputs: Inputs
    outputs: EncoderResult
    plan_results: Plans
    row_walks: tuple[str, ...]


def prepare(binding, resources):
    defaults = bind_default_call(binding, resources, input_type=Inputs, call_type=Call, plan_type=Plans)
    weights = prepare_weights(binding, "encoder.", dtype=torch.float32)
    encoder = WhisperEncoderB200(weights, TINY, max_batch=MAX_ROWS, device=binding.device)

    def run(call):  # enqueued on execution.stream by the device program
        features = torch.stack([f.to(binding.device, torch.float32) for f in call.inputs.audio_features])
        states = encoder(features)
        for owned, row in zip(call.outputs.encoder_states, states):
            owned.copy_(row)
        return {'encoder_states': call.outputs.encoder_states}

    # the reference's CPU helper refuses a CUDA binding; its device twin enqueues run()
    # and the owned-output copies on execution.stream. The encoder's device memory is
    # released if the binding fails (pi_cpu/audio_encoder.py:45-52).
    try:
        program = prepare_device_programs(binding, resources, {"prefill": DeviceProgram(run, slots=1)},
                                          call_binding=defaults)
    except BaseException:
        encoder.close()
        raise

    def close():
        program.close()
        encoder.close()
    return PreparedImplementation(program.materialize, program.primitive, program.acquire, close)


acceleration = Acceleration(
    reference=WhisperEncoderSubmodule,
    when=When(
        Eq('node_name', 'audio_encoder'),
        Eq('device_type', 'cuda'),
        SM100aAvailable(),
        Eq('dtype', torch.float32),
        When(Eq('graph_walk', 'prefill'), Eq('tp_size', 1), Eq('sp_size', 1)),
        Range('batch_size', 1, MAX_ROWS),
        Eq('config.d_model', 384),
        Eq('config.encoder_layers', 4),
        Eq('config.encoder_attention_heads', 6),
        Eq('config.encoder_ffn_dim', 1536),
        Eq('config.num_mel_bins', 80),
        Eq('config.max_source_positions', 1500),
        Eq('config.activation_function', 'gelu'),
    ),
    implementation=Implementation(prepare=prepare, resources=default_resource_requests),
)
