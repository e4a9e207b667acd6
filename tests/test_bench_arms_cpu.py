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
