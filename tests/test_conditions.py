"""The sm_100a Condition follows the reference's capability-gate contract
(cpu_ggml_q8.py:31-41): UNKNOWN without a binding, NO without the device,
a malformed deployment setting raises."""
from types import SimpleNamespace as NS

import pytest
import torch

from mstar_accelerators_b200.conditions import SM100aAvailable, Support, setting


def binding(device, config=None):
    return NS(device=torch.device(device), prepared={}, model_config=config or {})


def test_unknown_without_binding():
    cond = SM100aAvailable()
    assert cond.evaluate({}) is Support.UNKNOWN
    assert cond.specialize({}) is cond


def test_no_on_cpu_binding():
    cond = SM100aAvailable()
    assert cond.evaluate({"binding": binding("cpu")}) is Support.NO
    assert cond.specialize({"binding": binding("cpu")}).evaluate({}) is Support.NO


def test_cuda_binding_matches_device_capability():
    expect = torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
    got = SM100aAvailable().evaluate({"binding": binding("cuda")})
    assert got is (Support.YES if expect else Support.NO)


@pytest.mark.parametrize("value", [{"library": "relative.so", "sha256": "0" * 64},
                                   {"library": "/abs.so", "sha256": "ABC"},
                                   {"library": "/abs.so"}])
def test_malformed_setting_raises(value):
    with pytest.raises(ValueError):
        setting(binding("cuda", {"runtime_extension": {"b200": value}}))


def test_setting_round_trip():
    value = {"library": "/abs/libmstar_b200.so", "sha256": "a" * 64}
    assert setting(binding("cuda", {"runtime_extension": {"b200": value}})) == value
    assert setting(binding("cuda")) is None
