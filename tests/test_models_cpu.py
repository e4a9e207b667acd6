"""Model definitions on CPU (plain-PyTorch path): shapes, offload parity, rope tables."""

import torch

import flextensor_b200 as ft
from flextensor_b200.models.wan import WanDiT, init_wan_params_, rope_tables, tiny_config
from flextensor_b200.planner import NthLayerStrategy


def test_wan_tiny_forward_and_offload_parity():
    cfg = tiny_config()
    torch.manual_seed(0)
    m = WanDiT(cfg, impl="torch")
    init_wan_params_(m, seed=0)
    lat = torch.randn(1, cfg.in_channels, 2, 8, 8)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim)
    ts = torch.tensor([100.0])
    with torch.no_grad():
        ref = m(lat, ts, ctx)
    assert ref.shape == lat.shape and torch.isfinite(ref).all()
    om = ft.get_offload_manager()
    mm = om.offload(m, ft.OffloadConfig(pinned_memory=False, include_patterns=["blocks.*"], profiling_iters=1,
                                        num_blocks=2, min_blocks=2,
                                        load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True)))
    for _ in range(4):
        with torch.no_grad():
            assert torch.equal(mm(lat, ts, ctx), ref)
    assert om.phase.value == "inference"


def test_rope_table_splits():
    cos, sin = rope_tables((2, 3, 4), 128, "cpu")
    assert cos.shape == (24, 64)
    # first 22 pairs depend only on the frame index, the next 21 only on the row
    c = cos.view(2, 3, 4, 64)
    assert torch.allclose(c[:, :, :1, :22].expand(2, 3, 4, 22), c[..., :22])
    assert torch.allclose(c[:1, :, :1, 22:43].expand(2, 3, 4, 21), c[..., 22:43])
