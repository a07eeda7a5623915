"""Host logic of the tensor-parallel encoder (CPU): head and row ownership
splits, and the weight shards. Column shards (QKV by heads, fc1 rows) and row
shards (out_proj and fc2 columns) must reassemble the full matrices, cut only
at whole Q8_0 blocks, so each rank's packed blocks are exactly sub-blocks of the
single-GPU packing (checked with the oracle packer), and the sum of the
row-parallel partial products equals the full product.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O


def test_head_and_owner_splits():
    from mstar_accelerators_b200.encoder_tp import head_split, owner_split
    assert head_split(20, 8) == [3, 3, 3, 3, 2, 2, 2, 2]
    assert head_split(6, 2) == [3, 3]
    assert sum(head_split(20, 3)) == 20
    assert owner_split(24000, 8) == 3000 and owner_split(1500, 4) == 375 and owner_split(7, 2) == 4


@pytest.mark.parametrize("world", [2, 4])
def test_shards_reassemble_and_keep_blocks(world):
    from mstar_accelerators_b200.encoder import EncoderConfig, synthetic_weights
    from mstar_accelerators_b200.encoder_tp import shard_weights
    cfg = EncoderConfig(mels=80, width=256, heads=4, layers=1, positions=64)
    w = synthetic_weights(cfg, seed=2)
    shards = [shard_weights(w, cfg, world, r) for r in range(world)]
    p = "encoder.layers.0."
    for n in "qkv":
        full = w[p + f"self_attn.{n}_proj.weight"]
        assert torch.equal(torch.cat([s[p + f"self_attn.{n}_proj.weight"] for s in shards]), full)
    out_full = w[p + "self_attn.out_proj.weight"]
    assert torch.equal(torch.cat([s[p + "self_attn.out_proj.weight"] for s in shards], dim=1), out_full)
    fc2_full = w[p + "fc2.weight"]
    assert torch.equal(torch.cat([s[p + "fc2.weight"] for s in shards], dim=1), fc2_full)
    assert torch.equal(torch.cat([s[p + "fc1.bias"] for s in shards]), w[p + "fc1.bias"])
    # row-parallel shards are whole Q8_0 blocks of the full packing
    blocks = O.pack_weights(fc2_full.numpy()).reshape(cfg.width, -1, 34)
    k = cfg.ffn // world
    for r, s in enumerate(shards):
        part = O.pack_weights(s[p + "fc2.weight"].contiguous().numpy()).reshape(cfg.width, -1, 34)
        assert np.array_equal(part, blocks[:, r * k // 32:(r + 1) * k // 32])
    # the partial products sum to the full product
    x = np.random.default_rng(0).standard_normal((5, cfg.ffn))
    parts = sum(x[:, r * k:(r + 1) * k] @ s[p + "fc2.weight"].double().numpy().T for r, s in enumerate(shards))
    np.testing.assert_allclose(parts, x @ fc2_full.double().numpy().T, rtol=1e-12, atol=1e-12)


def test_shards_reject_unsplittable_geometry():
    from mstar_accelerators_b200.encoder import EncoderConfig, synthetic_weights
    from mstar_accelerators_b200.encoder_tp import shard_weights
    cfg = EncoderConfig(mels=80, width=96, heads=2, layers=1, positions=8)  # ffn 384 = 3 * 128
    w = synthetic_weights(cfg, seed=1)
    with pytest.raises(ValueError):
        shard_weights(w, cfg, 8, 0)
