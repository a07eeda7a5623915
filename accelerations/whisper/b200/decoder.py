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
from mstar_accelerators import Acceleration, AllRows, Eq, Implementation, Or, PreparedImplementation, Range, When
from mstar_accelerators.backends.weights import prepare_weights
from mstar_accelerators.compiler import bind_default_call
from mstar_accelerators.implementations.whisper.decoder_call import Call, Inputs, Plans, Resources
from mstar_accelerators_b200.conditions import SM100aAvailable
from mstar_accelerators_b200.programs import DeviceProgram, prepare_device_programs
from mstar_accelerators_b200.whisper import WhisperConfig, WhisperDecoderB200


def prepare(binding, resources):
    defaults = bind_default_call(binding, resources, input_type=Inputs, call_type=Call, plan_type=Plans)
    config = binding.submodule.config
    weights = prepare_weights(binding, defaults.contract.weight_prefix, dtype=torch.float32)
    suppressed = {walk: list(config.suppressed_tokens(walk)) for walk in ("prefill", "decode")}
    owners = {}

    def owner(rows):
        if rows not in owners:
            # every row brings its own encoder states, so each row has its own cross planes
            owners[rows] = WhisperDecoderB200(weights, WhisperConfig(), batch=rows, suppressed=suppressed,
                                              shared_cross=False, device=binding.device)
        return owners[rows]

    def run(call):
        ids = torch.stack([t.to(binding.device) for t in call.inputs.input_ids])
        dec = owner(ids.shape[0])
        if call.graph_walk == "prefill":
            enc = torch.stack([e for e in call.inputs.encoder_states if e is not None]).to(binding.device, torch.float32)
            _, tokens = dec.prefill(ids, enc)
        else:  # the position plan's rows follow the call's rows (cpu_ggml_decoder.py:213)
            positions = call.plan_results.positions["main"].to(binding.device).reshape(ids.shape[0], -1)[:, -1]
            _, tokens = dec.decode(ids.reshape(-1), positions)
        return {"tokens": tokens}

    # the reference's CPU helper refuses a CUDA binding; its device twin enqueues run()
    # and the owned-output copies on execution.stream
    program = prepare_device_programs(binding, resources,
                                      {walk: DeviceProgram(run) for walk in ("prefill", "decode")},
                                      call_binding=defaults)

    def close():
        program.close()
        for dec in owners.values():
            dec.close()
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
