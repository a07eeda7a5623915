"""The thinker prologue oracle (oracle/thinker_oracle.py, the reference's fused QK
RMSNorm + prepared MRoPE op, qknorm_rope.py:9-53) against the same formula in torch
float64 with the rotate_half of transformers' Qwen3-Omni attention: within one bf16
step (the oracle rounds at the reference's bf16 boundaries, the float64 form does
not), so the head layout, the rotation's sign and the cos / sin pairing are pinned."""
import numpy as np
import torch

from oracle import thinker_oracle as TO
from oracle.moe_oracle import bf16


def test_oracle_matches_float64_formula():
    rng = np.random.default_rng(0)
    T, Hq, Hk = 5, 32, 4
    q = bf16(rng.standard_normal((T, Hq, 128)) * 3)
    k = bf16(rng.standard_normal((T, Hk, 128)))
    qw, kw = bf16(1 + 0.1 * rng.standard_normal(128)), bf16(1 + 0.1 * rng.standard_normal(128))
    ang = rng.uniform(0, 50, (T, 64))
    cos = bf16(np.cos(np.concatenate([ang, ang], -1)))
    sin = bf16(np.sin(np.concatenate([ang, ang], -1)))
    oq, ok = TO.qknorm_rope(q, k, qw, kw, cos, sin, eps=1e-6)

    def ref(x, w):
        x = torch.from_numpy(x).double()
        n = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w).double()
        rot = torch.cat([-n[..., 64:], n[..., :64]], -1)     # transformers' rotate_half
        c, s = torch.from_numpy(cos).double()[:, None], torch.from_numpy(sin).double()[:, None]
        # bound: a few bf16 steps of the two products (their sum can cancel)
        return (n * c + rot * s).numpy(), (2 ** -6 * ((n * c).abs() + (rot * s).abs())).numpy() + 1e-6

    for got, (want, bound) in ((oq, ref(q, qw)), (ok, ref(k, kw))):
        assert np.all(np.abs(got - want) <= bound), np.abs(got - want).max()
