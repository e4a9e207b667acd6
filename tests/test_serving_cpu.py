"""HTTP serving path of the DiT example on the CPU (one rank, torch kernels, offloading on):
requests go through the rank-0 engine loop and the control plane and come back as JSON."""

import importlib.util
import os
import threading

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _load():
    spec = importlib.util.spec_from_file_location("ltx_serve", os.path.join(ROOT, "examples", "ltx_serving",
                                                                              "serve.py"))
    mod = importlib.util.module_from_spec(spec)
    import sys

    sys.modules[spec.name] = mod  # dataclasses resolve annotations through sys.modules
    spec.loader.exec_module(mod)
    return mod


def test_denoise_over_http():
    pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient

    import torch

    from flextensor_b200.models.wan import tiny_config
    from flextensor_b200.parallel.control import ControlPlane

    mod = _load()
    cfg = tiny_config(num_layers=2)
    engine = mod.DenoiseEngine(cfg, (2, 8, 8), torch.device("cpu"), impl="torch")
    loop = mod.Rank0Loop(engine, ControlPlane())
    stop = threading.Event()
    th = threading.Thread(target=loop.serve_forever, args=(stop,), daemon=True)
    th.start()
    try:
        client = TestClient(mod.make_app(loop.submit))
        assert client.get("/health").json() == {"ok": True}
        a = client.post("/denoise", json={"steps": 2, "seed": 3}).json()
        b = client.post("/denoise", json={"steps": 2, "seed": 3}).json()
        c = client.post("/denoise", json={"steps": 2, "seed": 4}).json()
        assert a["ok"] and a["steps"] == 2
        assert a["checksum"] == b["checksum"] != c["checksum"]
    finally:
        stop.set()
        th.join(5)


def test_profile_then_serve_from_profiles(tmp_path):
    """``profile`` saves one profile per stage manager (text encoder, DiT); ``serve`` restores both
    from them (no discovery / profiling) and answers a request; with ``--shm-namespace`` the
    stages come through a shared-memory session (this single process is the creator)."""
    import flextensor_b200 as ft

    mod = _load()
    pdir = str(tmp_path / "prof")
    saved = mod.main(["profile", "--profile-dir", pdir, "--tiny", "--cpu"])
    assert saved is None
    for stage in ("text", "dit"):
        assert os.path.exists(os.path.join(pdir, stage, "profile.json"))
        ft.release(stage)
    out = mod.main(["serve", "--profile-dir", pdir, "--tiny", "--cpu", "--once"])
    assert out["ok"] and out["steps"] == 2
    for stage in ("text", "dit"):
        assert ft.get_offload_manager(stage).phase.value == "inference"
        ft.release(stage)
    ns = f"ftserve_{os.getpid()}"
    out2 = mod.main(["serve", "--profile-dir", pdir, "--tiny", "--cpu", "--once", "--shm-namespace", ns])
    assert out2["ok"] and out2["checksum"] == out["checksum"]


def test_stage_config_uses_the_ranks_gpu():
    """Every rank's stage managers are configured for its own GPU, not the config's default 0."""
    import torch

    mod = _load()
    assert mod._stage_config("dit", 0.1, torch.device("cuda", 1)).gpu_device == 1
    assert mod._stage_config("text", None, torch.device("cuda", 0)).gpu_device == 0
    assert mod._stage_config("dit", None, torch.device("cpu")).gpu_device == 0
