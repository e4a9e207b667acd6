"""The two arms of ``bench.py``: same architecture, and a reference arm that runs no code of ours.

* ``baseline/wan_torch.py`` (the reference arm's workload, stock PyTorch ops only) has the
  parameter tree of ``flextensor_b200.models.wan.WanDiT`` and computes the same function as
  its plain-PyTorch path on the same weights.
* Importing the reference arm loads the reference package from ``baseline/_ref`` and never
  imports ``flextensor_b200`` (so none of this repository's native libraries can load).
"""

import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))

from wan_torch import WanShape, WanTorchDiT, init_params_  # noqa: E402

from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config  # noqa: E402


def _pair():
    cfg = tiny_config()
    ours = WanDiT(cfg, impl="torch").float()
    ref = WanTorchDiT(WanShape(**{k: getattr(cfg, k) for k in WanShape.__dataclass_fields__})).float()
    return cfg, ours, ref


def test_same_parameter_tree():
    _, ours, ref = _pair()
    a = {n: tuple(p.shape) for n, p in ours.named_parameters()}
    b = {n: tuple(p.shape) for n, p in ref.named_parameters()}
    assert a == b


def test_same_function_on_same_weights():
    cfg, ours, ref = _pair()
    init_wan_params_(ours, seed=3)
    ref.load_state_dict(ours.state_dict())
    torch.manual_seed(0)
    lat = torch.randn(1, cfg.in_channels, 2, 4, 6)
    ts = torch.tensor([321.0])
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim)
    with torch.no_grad():
        ya = ours(lat, ts, ctx)
        yb = ref(lat, ts, ctx)
    torch.testing.assert_close(yb, ya, rtol=1e-4, atol=1e-5)


def test_bf16_forward_matches_ours():
    cfg, ours, ref = _pair()
    init_wan_params_(ours, seed=4)
    ref.load_state_dict(ours.state_dict())
    ours, ref = ours.to(torch.bfloat16), ref.to(torch.bfloat16)
    torch.manual_seed(1)
    lat = torch.randn(1, cfg.in_channels, 2, 4, 6)
    ts = torch.tensor([500.0])
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim)
    with torch.no_grad():
        ya = ours(lat, ts, ctx).float()
        yb = ref(lat, ts, ctx).float()
    torch.testing.assert_close(yb, ya, rtol=2e-2, atol=2e-2)


def test_reference_init_is_seeded():
    _, _, ref = _pair()
    init_params_(ref, seed=5)
    w1 = ref.blocks[0].ffn_in.weight.clone()
    init_params_(ref, seed=5)
    assert torch.equal(w1, ref.blocks[0].ffn_in.weight)
    assert torch.all(ref.blocks[0].attn1.norm_q.weight == 1)


@pytest.mark.skipif(not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "flextensor")),
                    reason="reference not installed in baseline/_ref")
def test_reference_arm_imports_nothing_of_ours():
    code = (
        "import sys, bench\n"
        "ft, why = bench.import_arm('reference')\n"
        "assert ft is not None, why\n"
        "assert 'baseline/_ref' in ft.__file__.replace('\\\\', '/'), ft.__file__\n"
        "sys.path.insert(0, 'baseline')\n"
        "import wan_torch\n"
        "bad = [k for k in sys.modules if k.startswith('flextensor_b200')]\n"
        "assert not bad, bad\n"
        "print('OK')\n"
    )
    env = dict(os.environ, DISABLE_BEARTYPE="1")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


def _ulysses_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from wan_torch import Ulysses, WanShape, WanTorchDiT, init_params_

    torch.manual_seed(0)
    cfg = WanShape(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=128, text_len=16, freq_dim=64,
                   in_channels=16, out_channels=16, patch=(1, 1, 1))
    m = WanTorchDiT(cfg)
    init_params_(m, seed=2)
    lat = torch.randn(1, 16, 2, 4, 4, generator=torch.Generator().manual_seed(3))
    ctx = torch.randn(1, 16, 128, generator=torch.Generator().manual_seed(4))
    ts = torch.tensor([100.0])
    with torch.no_grad():
        want = m(lat, ts, ctx)
        got = m(lat, ts, ctx, cp=Ulysses())
    q.put((rank, float((got - want).abs().max())))
    dist.destroy_process_group()


def test_reference_ulysses_matches_unsharded_over_gloo():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_ulysses_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(30)
    assert all(err < 1e-4 for _, err in res), res


def _mixtral_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from llama_torch import rope_cos_sin
    from mixtral_torch import MixtralEP, MixtralShape, init_params_

    cfg = MixtralShape(dim=128, n_layers=2, n_heads=2, n_kv_heads=1, ffn_dim=64, n_experts=4, topk=2)
    cfg_head = cfg.head_dim
    full = MixtralEP(cfg, 0, 1)
    init_params_(full, seed=5)
    mine = MixtralEP(cfg, rank, world)
    el = cfg.n_experts // world
    with torch.no_grad():
        for lf, lm in zip(full.layers, mine.layers):
            for name, p in lm.named_parameters():
                if name.startswith("experts."):
                    j = int(name.split(".")[1])
                    p.copy_(lf.get_parameter(name.replace(f"experts.{j}.", f"experts.{rank * el + j}.")))
                else:
                    p.copy_(lf.get_parameter(name))
    B, S = 2, 8
    cos, sin = rope_cos_sin(S, cfg_head, cfg.rope_theta, "cpu")
    x = torch.randn(B * S, cfg.dim, generator=torch.Generator().manual_seed(rank))
    with torch.no_grad():
        want = full(x, B, S, cos, sin)
        got = mine(x, B, S, cos, sin)
    q.put((rank, float((got - want).abs().max())))
    dist.destroy_process_group()


def test_reference_mixtral_expert_parallel_matches_single_rank_over_gloo():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_mixtral_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(30)
    assert all(err < 1e-4 for _, err in res), res


def test_host_need_estimates():
    """Ours needs the streamed bytes once; the reference pays the pinned copies (power-of-two
    rounded) of every unit weight plus its packed streamed blocks."""
    import torch
    from torch import nn

    import bench

    with torch.device("meta"):
        m = nn.ModuleDict({"layers": nn.ModuleList([nn.Linear(1000, 1000, bias=False) for _ in range(4)]),
                           "head": nn.Linear(1000, 10, bias=False)})
    unit = 4 * 1000 * 1000 * 2   # counted as bf16
    assert bench.host_need_bytes(m, "ours", 0.5, "layers.") == unit // 2 + (2 << 30)
    per = 1 << (1000 * 1000 * 2 - 1).bit_length()
    assert bench.host_need_bytes(m, "reference", 0.5, "layers.") == 4 * per + unit // 2 + (2 << 30)


def test_host_start_bytes():
    import torch
    from torch import nn

    import bench

    with torch.device("meta"):
        m = nn.Linear(100, 10, bias=False)
    assert bench.host_start_bytes(m, "reference") == 100 * 10 * 2
    assert bench.host_start_bytes(m, "ours") == 0
