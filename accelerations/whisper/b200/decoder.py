"""B200 Whisper decoder: Q8_0 linears and Q4_0 readout on sm_100a kernels.

Same logical contract as accelerations/whisper/pi_cpu/decoder.py (reference
WhisperDecoderSubmodule, greedy readout with suppression, 4-token prefill and
1-token decode walks) gated by the sm_100a device Condition. Rows of one call
decode together: every GEMV row is one sequence (batch_size up to 32).

Requires the M* runtime (mstar); it is exercised through
python -m mstar_accelerators.testing --registry accelerations/whisper/b200.
"""
import torch

from mstar.model.whisper.submodules import WhisperDecoderSubmodule
from mstar_accelerators import Acceleration, AllRows, Eq, Implementation, Or, Range, When
from mstar_accelerators.backends.torch import TorchProgram, prepare_torch_programs
from mstar_accelerators.backends.weights import prepare_weights
from mstar_accelerators.compiler import bind_default_call
from mstar_accelerators.implementations.whisper.decoder_call import Call, Inputs, Plans, Resources
from mstar_accelerators_b200.conditions import SM100aAvailable
from mstar_accelerators_b200.whisper import WhisperConfig, WhisperDecoderB200


def prepare(binding, resources):
    defaults = bind_default_call(binding, resources, input_type=Inputs, call_type=Call, plan_type=Plans)
    config = binding.submodule.config
    weights = prepare_weights(binding, defaults.contract.weight_prefix, dtype=torch.float32)
    suppressed = {walk: list(config.suppressed_tokens(walk)) for walk in ("prefill", "decode")}
    owners = {}

    def owner(rows):
        if rows not in owners:
            owners[rows] = WhisperDecoderB200(weights, WhisperConfig(), batch=rows, suppressed=suppressed,
                                              device=binding.device)
        return owners[rows]

    def run(call):
        ids = torch.stack([t.to(binding.device) for t in call.inputs.input_ids])
        dec = owner(ids.shape[0])
        if call.graph_walk == "prefill":
            enc = torch.stack([e for e in call.inputs.encoder_states if e is not None])
            _, tokens = dec.prefill(ids, enc)
        else:
            positions = torch.stack([call.plan_results.positions[k] for k in sorted(call.plan_results.positions)])
            _, tokens = dec.decode(ids.reshape(-1), positions.reshape(-1).to(binding.device))
        return {"tokens": tokens}

    program = prepare_torch_programs(binding, resources,
                                     {walk: TorchProgram(run) for walk in ("prefill", "decode")},
                                     call_binding=defaults)

    def close():
        program.close()
        for dec in owners.values():
            dec.close()
    from mstar_accelerators import PreparedImplementation
    return PreparedImplementation(program.materialize, program.primitive, program.acquire, close)


acceleration = Acceleration(
    reference=WhisperDecoderSubmodule,
    when=When(
        Eq("node_name", "decoder"),
        Eq("device_type", "cuda"),
        SM100aAvailable(),
        Eq("dtype", torch.float32),
        Eq("tp_size", 1),
        Eq("sp_size", 1),
        Or(
            When(Eq("graph_walk", "decode"), AllRows(Resources.sampler, Eq("temperature", 0.0))),
            When(Eq("graph_walk", "prefill"), AllRows(Resources.sampler, Eq("temperature", 0.0))),
        ),
        Range("batch_size", 1, 32),
        Eq("config.d_model", 384),
        Eq("config.decoder_layers", 4),
        Eq("config.decoder_attention_heads", 6),
        Eq("config.decoder_ffn_dim", 1536),
        Eq("config.max_source_positions", 1500),
        Eq("config.max_target_positions", 448),
        Eq("config.vocab_size", 51865),
        Eq("config.activation_function", "gelu"),
        Eq("config.scale_embedding", False),
    ),
    implementation=Implementation(prepare=prepare),
)
