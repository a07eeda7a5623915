"""Selection logic of install_thinker_attention_linears (CPU, no kernels run).

Only plain nn.Linear projections named like the thinker's (q_proj, k_proj,
v_proj, qkv_proj, o_proj, lm_head) with a block-aligned input width are
targets; subclasses (tensor-parallel linears that own a collective) and other
names are left alone.
"""
from torch import nn

from mstar_accelerators_b200.thinker import thinker_linear_targets


class _Parallel(nn.Linear):
    pass


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(64, 128, bias=False)
        self.k_proj = nn.Linear(64, 32, bias=False)
        self.v_proj = nn.Linear(64, 32, bias=True)
        self.o_proj = _Parallel(128, 64)          # owns a collective in a TP build: not a target
        self.gate = nn.Linear(64, 8)              # other names are not targets


def test_targets_are_plain_named_projections():
    m = nn.Module()
    m.layers = nn.ModuleList([_Attn(), _Attn()])
    m.lm_head = nn.Linear(64, 1000, bias=False)
    m.odd = nn.Module()
    m.odd.q_proj = nn.Linear(40, 16)              # width not a multiple of 32
    names = [(p.__class__.__name__, n) for p, n, _ in thinker_linear_targets(m)]
    assert names.count(("_Attn", "q_proj")) == 2 and names.count(("_Attn", "v_proj")) == 2
    assert ("Module", "lm_head") in names
    assert all(n != "o_proj" and n != "gate" for _, n in names)
    assert len(names) == 7
