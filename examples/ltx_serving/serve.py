"""HTTP serving of a video DiT with weight offloading and context parallelism.

    python -m torch.distributed.run --nproc-per-node 8 examples/ltx_serving/serve.py --port 8000
    curl -X POST localhost:8000/denoise -d '{"steps": 4, "seed": 1}' -H 'content-type: application/json'

Every rank holds a replica of the LTX-shape DiT (``models/ltx.py``) with half of the weight
bytes offloaded (striped host streaming across the ranks) and runs its 1/N of the 40,480 latent
tokens (``ContextParallel``: the K/V all-gather is inside the attention kernel). Rank 0 serves
HTTP; each request is broadcast over the bounded Gloo control plane, all ranks run the denoise
steps, and the per-rank outcomes are exchanged before rank 0 answers; a failed or stalled rank
poisons the replica (``parallel/control.py``), which then refuses further requests.
Mirrors the reference's LTX serving example (``examples/ltx23/outpaint/serve_infer.py``).
"""

from __future__ import annotations

import argparse
import os
import queue
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


class DenoiseEngine:
    """Model + offload + CP state of one rank; ``run(request)`` executes one request."""

    def __init__(self, cfg, grid, device, cp=None, offload=True, budget: float = 0.5, impl: str = "fused"):
        import flextensor_b200 as ft
        from flextensor_b200.models.wan import WanDiT, init_wan_params_

        self.cfg, self.grid, self.device, self.cp = cfg, grid, device, cp
        model = WanDiT(cfg, impl=impl).to(device).to(torch.bfloat16 if device.type == "cuda" else torch.float32)
        init_wan_params_(model, seed=0)
        model.eval().requires_grad_(False)
        if offload:
            total = sum(p.numel() * p.element_size() for p in model.parameters())
            frac = None
            if device.type == "cuda":
                frac = budget * total / torch.cuda.get_device_properties(device).total_memory
            model = ft.offload(model, ft.OffloadConfig(
                include_patterns=["blocks.*"], num_blocks=2, min_blocks=2, max_gpu_mem_fraction=frac,
                profiling_iters=1, skip_discovery=True, pinned_memory=device.type == "cuda"), name="dit")
        self.model = model
        self.warm = False

    def run(self, req: dict) -> dict:
        steps = int(req.get("steps", 4))
        seed = int(req.get("seed", 0))
        f, h, w = self.grid
        g = torch.Generator(device=self.device).manual_seed(seed)
        dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        lat = torch.randn(1, self.cfg.in_channels, f, h, w, generator=g, device=self.device).to(dt)
        ctx = torch.randn(1, self.cfg.text_len, self.cfg.text_dim, generator=g, device=self.device).to(dt)
        t0 = time.perf_counter()
        with torch.no_grad():
            for i in range(steps):
                t = torch.tensor([1000.0 * (1 - i / max(1, steps))], device=self.device)
                v = self.model(lat, t, ctx, cp=self.cp) if self.cp is not None else self.model(lat, t, ctx)
                lat = (lat.float() - v.float() / max(1, steps)).to(dt)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return {"ok": True, "steps": steps, "seconds": round(time.perf_counter() - t0, 4),
                "checksum": float(lat.float().abs().mean())}


def make_app(submit):
    """FastAPI app; ``submit(request_dict) -> response_dict`` runs on the engine loop."""
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="flextensor_b200 DiT serving")

    @app.get("/health")
    def health():
        return {"ok": True}

    @app.post("/denoise")
    def denoise(req: dict):
        out = submit(req)
        if not out.get("ok"):
            raise HTTPException(status_code=503, detail=out.get("error", "replica failed"))
        return out

    return app


class Rank0Loop:
    """Requests from HTTP threads -> one engine loop that drives every rank."""

    def __init__(self, engine, control):
        self.engine, self.control = engine, control
        self.q: queue.Queue = queue.Queue()

    def submit(self, req: dict, timeout: float = 600.0) -> dict:
        box: dict = {}
        done = threading.Event()
        self.q.put((req, box, done))
        if not done.wait(timeout):
            return {"ok": False, "error": "request timed out"}
        return box["out"]

    def serve_forever(self, stop: threading.Event) -> None:
        while not stop.is_set():
            try:
                req, box, done = self.q.get(timeout=0.2)
            except queue.Empty:
                continue
            try:
                cmd = self.control.broadcast_object({"op": "denoise", **req})
                out = self.engine.run(cmd)
                if not self.control.request_ok(out):
                    out = {"ok": False, "error": f"replica poisoned: {self.control.poison_reason}"}
            except Exception as e:  # noqa: BLE001 - answer the client, keep the reason
                out = {"ok": False, "error": f"{type(e).__name__}: {e}"}
            box["out"] = out
            done.set()
        if not self.control.poisoned:
            self.control.broadcast_object({"op": "stop"})


def follower_loop(engine, control) -> None:
    while True:
        cmd = control.broadcast_object(None)
        if cmd.get("op") == "stop":
            return
        try:
            out = engine.run(cmd)
        except Exception as e:  # noqa: BLE001
            out = {"ok": False, "error": f"{type(e).__name__}: {e}"}
        control.request_ok(out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--control-timeout", type=float, default=600.0)
    a = ap.parse_args()
    import datetime

    import torch.distributed as dist

    from flextensor_b200.models.ltx import LTX_CP_CONFIG, LTX_LATENT_GRID
    from flextensor_b200.models.wan import WanConfig
    from flextensor_b200.parallel import enable_striped_streaming
    from flextensor_b200.parallel.control import ControlPlane
    from flextensor_b200.parallel.cp import ContextParallel

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    world = int(os.environ.get("WORLD_SIZE", 1))
    cp = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=a.control_timeout),
                                device_id=torch.device("cuda", local))
        enable_striped_streaming()
    cfg = WanConfig(**{**LTX_CP_CONFIG.__dict__, "num_layers": a.layers})
    f, h, w = LTX_LATENT_GRID
    if world > 1:
        cp = ContextParallel(f * h * w, kv_heads=cfg.num_heads)
    engine = DenoiseEngine(cfg, LTX_LATENT_GRID, torch.device("cuda", local), cp=cp)
    control = ControlPlane(timeout_seconds=a.control_timeout)
    if control.rank != 0:
        follower_loop(engine, control)
        return
    import uvicorn

    loop = Rank0Loop(engine, control)
    stop = threading.Event()
    server = uvicorn.Server(uvicorn.Config(make_app(loop.submit), host="127.0.0.1", port=a.port, log_level="info"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        loop.serve_forever(stop)
    except KeyboardInterrupt:
        stop.set()


if __name__ == "__main__":
    main()
