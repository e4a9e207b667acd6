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
