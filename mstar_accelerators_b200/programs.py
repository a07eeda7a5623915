"""Stream-ordered Torch programs on a CUDA binding.

The reference's ``prepare_torch_programs`` (src/mstar_accelerators/backends/
torch/programs.py:85-129) binds synchronous Torch callbacks to an explicit CPU
binding and refuses every other device (:95-96). ``prepare_device_programs`` is
its twin for a CUDA binding, with the same contract:

  * one pool of workspace leases per graph walk, ``DeviceProgram.slots`` leases
    each, or one shared ``capacity`` borrowed from the caller; ``acquire``
    returns None when the pool is full and raises once it is closed; a program
    with leases outstanding refuses to close (programs.py:23-82);
  * ``binding.services`` is asked to require the walks the mapping serves and
    walks outside ``binding.graph_walks`` are dropped (programs.py:97-101);
  * ``primitive(call, execution)`` runs the walk's callback, checks that it
    returned exactly the contract's output fields with the owned outputs'
    shapes, and copies each value into the call's owned output unless the
    callback already wrote that very tensor (programs.py:111-129).

What differs on a device: the callback and the owned-output copies are
enqueued on ``execution.stream`` (the worker's current Torch stream) instead of
running to completion on the host, so the outputs are complete at that stream's
completion boundary, which the device runtime's drain waits for
(backends/torch/device_runtime.py:24-28); a lease is closed by the engine at
that boundary, as for the CPU helper. Nothing here falls back to the CPU.
"""
from __future__ import annotations

import threading
from collections.abc import Callable, Mapping
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DeviceProgram:
    """A walk's callback, returning logical output fields (the reference's TorchProgram
    record, programs.py:15-20); ``slots`` leases unless a shared capacity is given."""

    run: Callable
    slots: int = 2


class WorkspaceCapacity:
    """Lease slots shared by the programs that borrow it (the reference's
    WorkspaceCapacity contract: positive slot count, close refused while leased)."""

    def __init__(self, slots: int = 1):
        if type(slots) is not int or slots < 1:
            raise ValueError("workspace capacity needs a positive integer slot count")
        self.slots, self.active, self.closed = slots, 0, False
        self.lock = threading.Lock()

    def close(self) -> None:
        with self.lock:
            if self.active:
                raise RuntimeError("workspace capacity still has acquired workspaces")
            self.closed = True


class _Lease:
    def __init__(self, pool: "_Pool"):
        self.pool, self.closed = pool, False

    def close(self) -> None:
        with self.pool.capacity.lock:
            if not self.closed:
                self.closed = True
                self.pool.active -= 1
                self.pool.capacity.active -= 1


class _Pool:
    def __init__(self, program, capacity=None):
        self.owns_capacity = capacity is None
        self.capacity = capacity if capacity is not None else WorkspaceCapacity(program.slots)
        self.program, self.active, self.closed = program, 0, False

    def acquire(self):
        with self.capacity.lock:
            if self.closed or self.capacity.closed:
                raise RuntimeError("device Torch program is closed")
            if self.capacity.active == self.capacity.slots:
                return None
            self.capacity.active += 1
            self.active += 1
            return _Lease(self)

    def close(self) -> None:
        with self.capacity.lock:
            if self.active:
                raise RuntimeError("device Torch program still has acquired workspaces")
            self.closed, self.program = True, None
            if self.owns_capacity:
                self.capacity.closed = True


def prepare_device_programs(binding, resources, programs: Mapping, *, call_binding=None, capacity=None):
    """Bind Torch callbacks that enqueue CUDA work to a CUDA binding (see the module text)."""
    from mstar_accelerators.compiler import bind_default_call
    from mstar_accelerators.conditions import In
    from mstar_accelerators.definition import PreparedImplementation

    device = torch.device(binding.device)
    if device.type != "cuda":
        raise ValueError("device Torch programs require a CUDA binding")
    if binding.services is not None:
        binding.services.require(In("graph_walk", tuple(programs)), origin="device Torch program mapping")
    if binding.graph_walks is not None:
        programs = {walk: program for walk, program in programs.items() if walk in binding.graph_walks}
    defaults = call_binding or bind_default_call(binding, resources)
    pools = {walk: _Pool(program, capacity) for walk, program in programs.items()}
    output_specs = tuple(defaults.contract.outputs)
    expected = frozenset(spec.name for spec in output_specs)

    def acquire(facts):
        return pools[facts.graph_walk].acquire()

    @torch.no_grad()
    def primitive(call, execution):
        lease = execution.workspace
        if lease.closed:
            raise RuntimeError("device Torch workspace has already been released")
        stream = getattr(execution, "stream", None) or torch.cuda.current_stream(device)
        with torch.cuda.stream(stream):
            values = lease.pool.program.run(call)
            if set(values) != expected:
                raise ValueError(f"Torch output fields differ: expected {sorted(expected)}, got {sorted(values)}")
            for spec in output_specs:
                destination = getattr(call.outputs, spec.name)
                source = values[spec.name]
                pairs = zip(destination, source, strict=True) if spec.per_request else ((destination, source),)
                for target, value in pairs:
                    if target.shape != value.shape:
                        raise ValueError(f"{spec.name}: expected {tuple(target.shape)}, got {tuple(value.shape)}")
                    if target is not value or type(target) is not torch.Tensor:
                        target.copy_(value, non_blocking=True)
        return defaults.result(call)

    def close():
        for pool in reversed(tuple(pools.values())):
            pool.close()

    return PreparedImplementation(defaults.materialize, primitive, acquire, close)
