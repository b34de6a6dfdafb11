"""ShrimpNet module contract on CPU: parameter names, shapes, counts, seeded
init, and the refusal to run without CUDA tensors."""

from __future__ import annotations

import pytest
import torch

from hexo_bot_b200 import constants as K
from hexo_bot_b200.model import ShrimpNet, infer_net_kwargs_from_state_dict
from hexo_bot_b200.plugin import get_plugin


def test_param_count_default_env():
    # reference tests/test_shrimp_model.py:60-62 (C=96, 4 heads, CCCACCCACCA)
    assert sum(p.numel() for p in ShrimpNet().parameters()) == 1_656_453


@pytest.mark.parametrize(
    "kw,count",
    [
        (dict(channels=32, attention_heads=4, trunk_layout="CCA"), 93_533),
        (dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA"), 3_053_609),
        (dict(channels=192, attention_heads=12, trunk_layout="CCACCACCACCA"), 6_804_345),
    ],
)
def test_param_counts_bench_configs(kw, count):
    assert sum(p.numel() for p in ShrimpNet(**kw).parameters()) == count


def test_state_dict_layout():
    sd = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA").state_dict()
    assert sd["stem.weight"].shape == (7, 15, 32)
    assert sd["conv_blocks.1.conv2.weight"].shape == (7, 32, 32)
    assert sd["attn_blocks.0.attn.q_proj.weight"].shape == (32, 32)
    assert sd["attn_blocks.0.fc1.weight"].shape == (64, 32)
    assert sd["bias_tables.0"].shape == (K.BIAS_ROWS, 4)
    assert sd["tokens"].shape == (8, 32)
    assert sd["value_reduction.weight"].shape == (32, 96)
    assert sd["value_head.weight"].shape == (65, 32)
    assert "_cell_bias_lut_u8" not in sd


def test_fresh_model_init_contract():
    # reference tests/test_shrimp_model.py:288-314
    torch.manual_seed(7)
    m = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA")
    for blk in m.conv_blocks:
        assert torch.equal(blk.ls.gamma, torch.full((32,), 1e-4))
    for blk in m.attn_blocks:
        assert torch.equal(blk.ls_attn.gamma, torch.full((32,), 1e-4))
        assert torch.equal(blk.ls_mlp.gamma, torch.full((32,), 1e-4))
    for t in m.bias_tables:
        assert torch.count_nonzero(t).item() == 0


def test_infer_kwargs_roundtrip():
    sd = ShrimpNet(channels=64, attention_heads=4, trunk_layout="CCCACCCACCA").state_dict()
    assert infer_net_kwargs_from_state_dict(sd) == {"channels": 64, "attention_heads": 4,
                                                    "trunk_layout": "CCCACCCACCA"}


def test_strict_load_between_instances():
    a = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA")
    b = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA")
    b.load_state_dict(a.state_dict(), strict=True)
    for (ka, va), (kb, vb) in zip(a.state_dict().items(), b.state_dict().items()):
        assert ka == kb and torch.equal(va, vb)


def test_invalid_layouts_rejected():
    for bad in ("", "CCX", "CAC"):
        with pytest.raises(ValueError):
            ShrimpNet(channels=32, attention_heads=4, trunk_layout=bad)


def test_cpu_inputs_raise():
    m = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA")
    feats = torch.zeros(1, 7, 15)
    nbr = torch.full((1, 7, 6), 7)
    mask = torch.ones(1, 7, dtype=torch.bool)
    coords = torch.zeros(1, 7, 2, dtype=torch.long)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m.forward_policy_value(feats, nbr, mask, coords)
    with pytest.raises(NotImplementedError):
        m(feats, nbr, mask, coords)


def test_plugin_builds_model():
    net = get_plugin().build_model({}, {})
    assert isinstance(net, ShrimpNet)
    assert net.channels == K.CHANNELS


def test_kernel_launch_count():
    assert ShrimpNet.kernel_launches("CCACCACCACCA") == 2 + 1 + 16 + 16 + 2
    assert ShrimpNet.kernel_launches("CCACCACCACCA", channels=192) == 2 + 1 + 16 + 20 + 2
    assert ShrimpNet.kernel_launches("CCACCACCACCA", grid=True) == 2 + 1 + 1 + 16 + 9 + 16 + 2
    # small batches of long positions pool the heads' cell mean in a kernel of their own
    assert ShrimpNet.kernel_launches("CCACCACCACCA", pooled=True) == 2 + 1 + 16 + 16 + 2 + 1
    assert ShrimpNet.pools_cells_apart(6, 2432) and ShrimpNet.pools_cells_apart(588, 129)
    assert not ShrimpNet.pools_cells_apart(589, 129)  # 148 heads CTAs: one per SM
    assert not ShrimpNet.pools_cells_apart(3, 128)  # one chunk of cells
