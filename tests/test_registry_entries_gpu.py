"""The B200 Whisper registry entries, prepared and run on a CUDA binding.

The M* runtime (``mstar``) and the reference package are absent here, so the
modules an entry imports are replaced by small stand-ins (the stub pattern of
tests/golden/make_golden.py): the registry records (Acceleration, When, Eq, ...)
only hold their arguments, ``bind_default_call`` returns a contract with the
node's output fields, ``prepare_weights`` returns the synthetic checkpoint under
the node's prefix. Everything below the entry is the real code: the entry's
``prepare`` builds the B200 encoder / decoder, binds it through
``prepare_device_programs`` (the CUDA twin of the reference's CPU-only
prepare_torch_programs), and ``acquire`` + ``primitive`` run one call on a side
stream into owned output tensors, which are then compared with the oracle.
"""
import importlib.util
import sys
import types
from dataclasses import dataclass, field
from pathlib import Path
from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


class _Record:
    def __init__(self, *args, **kwargs):
        self.args, self.kwargs = args, kwargs


@dataclass(frozen=True)
class _Prepared:
    materialize: object
    primitive: object
    acquire: object
    close: object


@dataclass(frozen=True)
class _Implementation:
    prepare: object = None
    resources: object = field(default_factory=dict)
    cost: object = None
    execution: object = None


@dataclass(frozen=True)
class _Acceleration:
    reference: type
    when: object
    implementation: _Implementation


@dataclass(frozen=True)
class _Spec:
    name: str
    per_request: bool


def _contract(outputs, prefix):
    def bind(binding, resources, **types_):
        return NS(contract=NS(outputs=outputs, weight_prefix=prefix), materialize=lambda *a, **k: None,
                  result=lambda call: call.outputs, types=types_)
    return bind


def install_stubs(monkeypatch, weights, outputs, prefix):
    def mod(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        monkeypatch.setitem(sys.modules, name, m)
        return m

    @dataclass(frozen=True)
    class EncoderResult:
        encoder_states: tuple

    for name in ("mstar", "mstar.model", "mstar.model.whisper", "mstar_accelerators.backends",
                 "mstar_accelerators.implementations", "mstar_accelerators.implementations.whisper"):
        mod(name)
    mod("mstar.model.whisper.results", EncoderResult=EncoderResult)
    mod("mstar.model.whisper.submodules", WhisperEncoderSubmodule=type("WhisperEncoderSubmodule", (), {}),
        WhisperDecoderSubmodule=type("WhisperDecoderSubmodule", (), {}))
    mod("mstar_accelerators", Acceleration=_Acceleration, Implementation=_Implementation,
        PreparedImplementation=_Prepared, When=_Record, Eq=_Record, Range=_Record, Or=_Record, AllRows=_Record)
    mod("mstar_accelerators.backends.weights",
        prepare_weights=lambda binding, pre, dtype=None: {k: v.to(dtype) for k, v in weights.items()
                                                          if k.startswith(pre)})
    mod("mstar_accelerators.compiler", bind_default_call=_contract(outputs, prefix),
        default_resource_requests=lambda binding: {})
    mod("mstar_accelerators.conditions", In=_Record)
    mod("mstar_accelerators.definition", PreparedImplementation=_Prepared)
    mod("mstar_accelerators.implementations.whisper.decoder_call", Call=object, Inputs=object, Plans=object,
        Resources=NS(sampler="sampler"))


def load_entry(monkeypatch, name):
    spec = importlib.util.spec_from_file_location(f"_b200_entry_{name[:-3]}", ROOT / "accelerations/whisper/b200" / name)
    module = importlib.util.module_from_spec(spec)
    monkeypatch.setitem(sys.modules, spec.name, module)   # dataclasses resolve annotations through it
    spec.loader.exec_module(module)
    return module


def binding_for(submodule=None):
    return NS(device=torch.device("cuda", torch.cuda.current_device()), services=None, graph_walks=None,
              submodule=submodule, prepared={})


def test_audio_encoder_entry_prepares_and_runs_on_cuda(monkeypatch):
    from mstar_accelerators_b200.encoder import TINY, synthetic_mel, synthetic_weights
    from oracle import whisper_encoder_oracle as EO
    weights = synthetic_weights(TINY, seed=1)
    install_stubs(monkeypatch, weights, [_Spec("encoder_states", True)], "encoder.")
    entry = load_entry(monkeypatch, "audio_encoder.py")
    prepared = entry.acceleration.implementation.prepare(binding_for(), {})
    mel = synthetic_mel(TINY, 2, seed=2)
    owned = tuple(torch.full((1500, 384), float("nan"), device="cuda") for _ in range(2))
    call = entry.Call(graph_walk="prefill", inputs=entry.Inputs(audio_features=(mel[0], mel[1])),
                      outputs=NS(encoder_states=owned), plan_results=entry.Plans(), row_walks=("prefill",) * 2)
    lease = prepared.acquire(NS(graph_walk="prefill"))
    assert lease is not None and prepared.acquire(NS(graph_walk="prefill")) is None  # one slot
    stream = torch.cuda.Stream()
    result = prepared.primitive(call, NS(stream=stream, workspace=lease))
    stream.synchronize()
    assert result is call.outputs
    with pytest.raises(RuntimeError):
        prepared.close()     # a lease is still out
    lease.close()
    prepared.close()
    got = torch.stack(owned).cpu().numpy()
    ref = EO.WhisperEncoderOracle({k: v.numpy() for k, v in weights.items()}, TINY, "arm").forward(mel.numpy())
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 3e-2 * scale and np.abs(got - ref).mean() <= 3e-3 * scale


def test_decoder_entry_prefill_and_decode_on_cuda(monkeypatch):
    from mstar_accelerators_b200.whisper import WhisperConfig, synthetic_weights
    from oracle.whisper_oracle import WhisperDecoderOracle
    cfg = WhisperConfig()
    weights = synthetic_weights(cfg, seed=1)
    install_stubs(monkeypatch, weights, [_Spec("tokens", False)], "decoder.")
    entry = load_entry(monkeypatch, "decoder.py")
    sup = {"prefill": [50257, 220], "decode": [50257]}
    submodule = NS(config=NS(suppressed_tokens=lambda walk: sup[walk]))
    prepared = entry.acceleration.implementation.prepare(binding_for(submodule), {})
    B = 2
    enc = torch.randn((B, cfg.source, cfg.d_model), generator=torch.Generator().manual_seed(2))
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, (B, 4))
    ref = WhisperDecoderOracle(weights, cfg, batch=B, suppressed=sup)
    ref.set_cross(enc.numpy())
    stream = torch.cuda.Stream()
    tokens = torch.zeros(B, dtype=torch.int64, device="cuda")

    def run(walk, ids, positions, encoder):
        call = NS(graph_walk=walk, inputs=NS(input_ids=tuple(torch.from_numpy(r) for r in ids),
                                             encoder_states=encoder),
                  outputs=NS(tokens=tokens), plan_results=NS(positions={"main": torch.from_numpy(positions)}),
                  row_walks=(walk,) * B)
        lease = prepared.acquire(NS(graph_walk=walk))
        prepared.primitive(call, NS(stream=stream, workspace=lease))
        stream.synchronize()
        lease.close()
        return tokens.cpu().numpy().copy()

    got = run("prefill", prompt, np.tile(np.arange(4), B), tuple(enc))
    _, want = ref.forward(prompt, np.tile(np.arange(4), (B, 1)), "prefill")
    assert np.array_equal(got, want), (got, want)
    for step in range(3):
        pos = 4 + step
        got = run("decode", want[:, None], np.full(B, pos), ())
        _, nxt = ref.forward(want[:, None], np.full((B, 1), pos), "decode")
        assert np.array_equal(got, nxt), (step, got, nxt)
        want = nxt
    prepared.close()

