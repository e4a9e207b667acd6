"""One tiny end-to-end step of the flagship path: a 2-block Wan-shape DiT on the
fused sm_100a kernels, offloaded through the streaming runtime (profiling ->
plan -> ring-slot inference), checked against the plain-PyTorch path."""

from __future__ import annotations

import torch


def run_smoke(device: torch.device) -> dict:
    import flextensor_b200 as ft
    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
    from flextensor_b200.ops import native

    cfg = tiny_config()
    torch.manual_seed(0)
    model = WanDiT(cfg, impl="fused").to(torch.bfloat16)
    init_wan_params_(model, seed=0)
    ref = WanDiT(cfg, impl="torch").to(torch.bfloat16)
    ref.load_state_dict(model.state_dict())
    ref = ref.to(device)
    lat = torch.randn(1, cfg.in_channels, 2, 16, 16, device=device, dtype=torch.bfloat16)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=device, dtype=torch.bfloat16)
    ts = torch.tensor([321.0], device=device)
    with torch.no_grad():
        want = ref(lat, ts, ctx).float()
    om = ft.get_offload_manager("smoke")
    cfg_o = ft.OffloadConfig(gpu_device=device.index or 0, include_patterns=["blocks.*"], skip_discovery=True,
                             profiling_iters=1, num_blocks=2, min_blocks=2,
                             load_strategy=ft.NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    m = om.offload(model, cfg_o)
    with torch.no_grad():
        outs = [m(lat, ts, ctx).float() for _ in range(3)]
    torch.cuda.synchronize(device)
    err = native.device_error(reset=True)
    rel = max(((o - want).norm() / want.norm()).item() for o in outs)
    phase = om.phase.value
    om.release()
    if err != 0 or not all(torch.isfinite(o).all() for o in outs) or rel > 5e-2 or phase != "inference":
        raise RuntimeError(f"smoke failed: device_error={err} rel_err={rel:.3e} phase={phase}")
    return {"rel_err": rel, "phase": phase}
