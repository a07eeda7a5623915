"""Host logic of prepare_device_programs (the CUDA twin of the reference's
prepare_torch_programs, backends/torch/programs.py:85-129), on the CPU with the
reference's registry modules stubbed: the device check, the services
requirement, the graph-walk filter, and the lease pools (slots, a full pool
answers None, close refused while a lease is out, a closed pool refuses leases,
a borrowed capacity shared by two walks)."""
import sys
import types
from types import SimpleNamespace as NS

import pytest
import torch


@pytest.fixture
def programs(monkeypatch):
    class In:
        def __init__(self, *args):
            self.args = args

    def mod(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        monkeypatch.setitem(sys.modules, name, m)

    mod("mstar_accelerators")
    mod("mstar_accelerators.compiler", bind_default_call=lambda b, r, **k: NS(
        contract=NS(outputs=[NS(name="tokens", per_request=False)]), materialize=None, result=lambda c: c))
    mod("mstar_accelerators.conditions", In=In)
    mod("mstar_accelerators.definition", PreparedImplementation=lambda *a: NS(
        materialize=a[0], primitive=a[1], acquire=a[2], close=a[3]))
    from mstar_accelerators_b200 import programs
    return programs


def cuda_binding(**kw):
    return NS(device=torch.device("cuda", 0), services=kw.get("services"), graph_walks=kw.get("walks"))


def test_refuses_a_cpu_binding(programs):
    cpu = NS(device=torch.device("cpu"), services=None, graph_walks=None)
    with pytest.raises(ValueError):
        programs.prepare_device_programs(cpu, {}, {"decode": programs.DeviceProgram(lambda c: {})})


def test_services_requirement_and_walk_filter(programs):
    seen = []
    services = NS(require=lambda cond, origin: seen.append(cond.args))
    p = programs.prepare_device_programs(cuda_binding(services=services, walks=("decode",)), {},
                                         {"prefill": programs.DeviceProgram(lambda c: {}),
                                          "decode": programs.DeviceProgram(lambda c: {})})
    assert seen == [("graph_walk", ("prefill", "decode"))]
    assert p.acquire(NS(graph_walk="decode")) is not None
    with pytest.raises(KeyError):
        p.acquire(NS(graph_walk="prefill"))


def test_lease_pools(programs):
    p = programs.prepare_device_programs(cuda_binding(), {}, {"decode": programs.DeviceProgram(lambda c: {}, slots=2)})
    a, b = p.acquire(NS(graph_walk="decode")), p.acquire(NS(graph_walk="decode"))
    assert a is not None and b is not None and p.acquire(NS(graph_walk="decode")) is None
    a.close()
    a.close()   # idempotent
    with pytest.raises(RuntimeError):
        p.close()
    b.close()
    p.close()
    with pytest.raises(RuntimeError):
        p.acquire(NS(graph_walk="decode"))


def test_shared_capacity(programs):
    cap = programs.WorkspaceCapacity(1)
    p = programs.prepare_device_programs(cuda_binding(), {}, {"prefill": programs.DeviceProgram(lambda c: {}),
                                                             "decode": programs.DeviceProgram(lambda c: {})},
                                         capacity=cap)
    lease = p.acquire(NS(graph_walk="prefill"))
    assert p.acquire(NS(graph_walk="decode")) is None
    with pytest.raises(RuntimeError):
        cap.close()
    lease.close()
    p.close()
    assert not cap.closed   # borrowed: its owner closes it
    cap.close()
    with pytest.raises(ValueError):
        programs.WorkspaceCapacity(0)
