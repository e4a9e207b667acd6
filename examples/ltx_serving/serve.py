"""HTTP serving of a video DiT with weight offloading, shared host weights and context parallelism.

Two steps, as in the reference's LTX example (``examples/ltx23/outpaint/serve_infer.py``):

    # 1. build the stages, run the discovery / profiling passes, save one profile per manager
    python examples/ltx_serving/serve.py profile --profile-dir /tmp/ltx_profile

    # 2. serve from the saved profiles (one replica per GPU group)
    python -m torch.distributed.run --nproc-per-node 8 examples/ltx_serving/serve.py serve \\
        --profile-dir /tmp/ltx_profile --port 8000
    curl -X POST localhost:8000/denoise -d '{"steps": 4, "seed": 1}' -H 'content-type: application/json'

Stages, each under its own FlexTensor manager:

* ``text``: a transformer text encoder (token ids -> the DiT's context);
* ``dit``: the LTX-shape DiT (``models/ltx.py``), with half of its weight bytes streamed.

``serve`` restores both stages from the saved profiles without discovery or profiling. Running
several replicas on one node (e.g. 8 single-GPU replicas behind the ``nginx.conf`` next to this
file, or 4 CP2 replicas), ``--shm-namespace`` makes them share ONE host copy of the streamed
weights: the first replica loads the weights and publishes them in POSIX shared memory, and the
others build their models on the meta device and attach (``SharedOffloadSession``).

Within a replica of N GPUs (``torch.distributed.run --nproc-per-node N``), every rank runs
1/N of the 40,480 latent tokens (``ContextParallel``: the K/V all-gather is inside the attention
kernel) and streams 1/N of every offloaded block over its own PCIe link (striped streaming).
Rank 0 serves HTTP; each request goes to every rank over the bounded Gloo control plane, and
the per-rank outcomes are exchanged before rank 0 answers. A failed or stalled rank poisons the
replica (``parallel/control.py``), which then refuses further requests.
"""

from __future__ import annotations

import argparse
import contextlib
import os
import queue
import sys
import threading
import time
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


# ----------------------------------------------------------------------------- text stage
@dataclass
class TextConfig:
    vocab: int = 32000
    dim: int = 2048
    heads: int = 16
    layers: int = 8
    out_dim: int = 4096  # the DiT's text_dim
    max_len: int = 512


class _TextBlock(nn.Module):
    def __init__(self, c: TextConfig):
        super().__init__()
        self.heads = c.heads
        self.norm1 = nn.LayerNorm(c.dim)
        self.qkv = nn.Linear(c.dim, 3 * c.dim)
        self.proj = nn.Linear(c.dim, c.dim)
        self.norm2 = nn.LayerNorm(c.dim)
        self.fc1 = nn.Linear(c.dim, 4 * c.dim)
        self.fc2 = nn.Linear(4 * c.dim, c.dim)

    def forward(self, x):
        B, L, D = x.shape
        q, k, v = self.qkv(self.norm1(x)).view(B, L, 3, self.heads, D // self.heads).unbind(2)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        x = x + self.proj(o.transpose(1, 2).reshape(B, L, D))
        return x + self.fc2(F.gelu(self.fc1(self.norm2(x)), approximate="tanh"))


class TextEncoder(nn.Module):
    """Token ids ``[B, L]`` -> context ``[B, L, out_dim]`` (random-init; the offload units are
    ``blocks.*``)."""

    def __init__(self, c: TextConfig):
        super().__init__()
        self.cfg = c
        self.embed = nn.Embedding(c.vocab, c.dim)
        self.pos = nn.Parameter(torch.zeros(1, c.max_len, c.dim))
        self.blocks = nn.ModuleList([_TextBlock(c) for _ in range(c.layers)])
        self.norm = nn.LayerNorm(c.dim)
        self.out = nn.Linear(c.dim, c.out_dim)

    def forward(self, ids):
        x = self.embed(ids) + self.pos[:, :ids.shape[1]]
        for b in self.blocks:
            x = b(x)
        return self.out(self.norm(x))


def init_text_params_(m: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    g = torch.Generator(device=next(m.parameters()).device)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name:
                p.fill_(1.0 if name.endswith("weight") else 0.0)
            else:
                p.normal_(0.0, std, generator=g)


# ----------------------------------------------------------------------------- stages
STAGES = ("text", "dit")


def _stage_config(name: str, budget: float | None, device: torch.device):
    import flextensor_b200 as ft

    include = ["blocks.*"]
    # every rank's managers run on its own GPU (the config's default device is GPU 0)
    return ft.OffloadConfig(include_patterns=include, num_blocks=2, min_blocks=2, max_gpu_mem_fraction=budget,
                            profiling_iters=1, discovery_iters=1, pinned_memory=device.type == "cuda",
                            gpu_device=(device.index or 0) if device.type == "cuda" else 0)


class DenoiseEngine:
    """Model stages + offload + CP state of one rank; ``run(request)`` executes one request.

    ``mode``: ``offload`` (profile on the first requests, the historical single-step form),
    ``profile`` (offload with discovery / profiling; ``save_profiles`` writes them) or ``serve``
    (restore every stage from ``profile_dir``; with ``session`` through shared host memory)."""

    def __init__(self, cfg, grid, device, cp=None, offload=True, budget: float = 0.5, impl: str = "fused",
                 text_cfg: TextConfig | None = None, mode: str = "offload", profile_dir: str | None = None,
                 session=None, dit_dtype: torch.dtype | None = None):
        self.cfg, self.grid, self.device, self.cp = cfg, grid, device, cp
        self.impl, self.mode, self.profile_dir, self.session = impl, mode, profile_dir, session
        self.dtype = dit_dtype or (torch.bfloat16 if device.type == "cuda" else torch.float32)
        self.text_cfg = text_cfg
        self.offload_on = offload
        self.budget = budget
        self.model = self._stage("dit", self._build_dit, self._dit_bytes())
        self.text = self._stage("text", self._build_text, None) if text_cfg is not None else None

    # model factories (real weights, or a meta skeleton for shared-memory followers)
    def _build_dit(self, meta: bool = False):
        from flextensor_b200.models.wan import WanDiT, init_wan_params_

        if meta:
            with torch.device("meta"):
                return WanDiT(self.cfg, impl=self.impl).to(self.dtype).eval().requires_grad_(False)
        m = WanDiT(self.cfg, impl=self.impl).to(self.device).to(self.dtype)
        init_wan_params_(m, seed=0)
        return m.eval().requires_grad_(False)

    def _build_text(self, meta: bool = False):
        if meta:
            with torch.device("meta"):
                return TextEncoder(self.text_cfg).to(self.dtype).eval().requires_grad_(False)
        m = TextEncoder(self.text_cfg).to(self.device)
        init_text_params_(m, seed=1)
        return m.to(self.dtype).eval().requires_grad_(False)

    def _dit_bytes(self) -> int:
        c = self.cfg
        per_block = 2 * (8 * c.dim * c.dim + 2 * c.dim * c.ffn_dim)
        return per_block * c.num_layers

    def _stage(self, name: str, build, nbytes: int | None):
        import flextensor_b200 as ft

        frac = None
        if self.device.type == "cuda" and nbytes:
            frac = self.budget * nbytes / torch.cuda.get_device_properties(self.device).total_memory
        cfg = _stage_config(name, frac, self.device)
        if not self.offload_on:
            return build()
        if self.mode == "serve":
            pdir = os.path.join(self.profile_dir, name)
            if self.session is not None:
                return self.session.offload_from_profile(pdir, config=cfg, name=name,
                                                         creator_model_factory=build,
                                                         follower_model_factory=lambda: build(meta=True),
                                                         materialize_device=self.device)
            return ft.offload_from_profile(build(), pdir, config=cfg, name=name)
        return ft.offload(build(), cfg, name=name)

    def save_profiles(self) -> list[str]:
        import flextensor_b200 as ft

        saved = []
        for name in STAGES:
            if name == "text" and self.text is None:
                continue
            d = os.path.join(self.profile_dir, name)
            os.makedirs(d, exist_ok=True)
            ft.save_profile(d, name=name)
            saved.append(d)
        return saved

    def passes_needed(self) -> int:
        import flextensor_b200 as ft

        return max(ft.get_offload_manager(n).iters_before_inference for n in STAGES
                   if n == "dit" or self.text is not None)

    def _context(self, g, req: dict):
        c = self.cfg
        if self.text is None:
            return torch.randn(1, c.text_len, c.text_dim, generator=g, device=self.device).to(self.dtype)
        ids = req.get("prompt_ids")
        if ids is None:
            ids = torch.randint(0, self.text_cfg.vocab, (1, c.text_len), generator=g, device=self.device)
        else:
            ids = torch.tensor([list(ids)[:self.text_cfg.max_len]], device=self.device)
        with torch.no_grad():
            return self.text(ids).to(self.dtype)

    def run(self, req: dict) -> dict:
        steps = int(req.get("steps", 4))
        seed = int(req.get("seed", 0))
        f, h, w = self.grid
        g = torch.Generator(device=self.device).manual_seed(seed)
        lat = torch.randn(1, self.cfg.in_channels, f, h, w, generator=g, device=self.device).to(self.dtype)
        ctx = self._context(g, req)
        t0 = time.perf_counter()
        with torch.no_grad():
            for i in range(steps):
                t = torch.tensor([1000.0 * (1 - i / max(1, steps))], device=self.device)
                v = self.model(lat, t, ctx, cp=self.cp) if self.cp is not None else self.model(lat, t, ctx)
                lat = (lat.float() - v.float() / max(1, steps)).to(self.dtype)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return {"ok": True, "steps": steps, "seconds": round(time.perf_counter() - t0, 4),
                "checksum": float(lat.float().abs().mean())}


# ----------------------------------------------------------------------------- HTTP + control plane
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


# ----------------------------------------------------------------------------- entry points
def _shapes(a):
    from flextensor_b200.models.ltx import LTX_CP_CONFIG, LTX_LATENT_GRID
    from flextensor_b200.models.wan import WanConfig, tiny_config

    if a.tiny:  # CPU / smoke shapes
        return tiny_config(num_layers=2), (2, 8, 8), TextConfig(vocab=512, dim=64, heads=4, layers=2, out_dim=128,
                                                              max_len=64)
    cfg = WanConfig(**{**LTX_CP_CONFIG.__dict__, "num_layers": a.layers})
    return cfg, LTX_LATENT_GRID, TextConfig(out_dim=cfg.text_dim, max_len=cfg.text_len)


def _device(a):
    if a.cpu or not torch.cuda.is_available():
        return torch.device("cpu")
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    return torch.device("cuda", local)


def cmd_profile(a) -> list[str]:
    """Build the stages, drive the discovery / profiling passes, save one profile per manager."""
    cfg, grid, tcfg = _shapes(a)
    dev = _device(a)
    engine = DenoiseEngine(cfg, grid, dev, impl="fused" if dev.type == "cuda" else "torch",
                           text_cfg=tcfg if a.text_stage else None, mode="profile", profile_dir=a.profile_dir)
    for i in range(engine.passes_needed() + 1):
        engine.run({"steps": 1, "seed": i})
    return engine.save_profiles()


def cmd_serve(a):
    import datetime

    import torch.distributed as dist

    from flextensor_b200.parallel import enable_striped_streaming
    from flextensor_b200.parallel.control import ControlPlane
    from flextensor_b200.parallel.cp import ContextParallel
    from flextensor_b200.shared_offload import SharedOffloadSession

    cfg, grid, tcfg = _shapes(a)
    dev = _device(a)
    world = int(os.environ.get("WORLD_SIZE", 1))
    cp = None
    if world > 1:
        dist.init_process_group("nccl" if dev.type == "cuda" else "gloo",
                                timeout=datetime.timedelta(seconds=a.control_timeout),
                                device_id=dev if dev.type == "cuda" else None)
        if dev.type == "cuda":
            enable_striped_streaming()
            f, h, w = grid
            cp = ContextParallel((f // cfg.patch[0]) * (h // cfg.patch[1]) * (w // cfg.patch[2]),
                                 kv_heads=cfg.num_heads)
    session_cm = (SharedOffloadSession(a.shm_namespace, wait_timeout=a.shm_wait_timeout) if a.shm_namespace
                  else contextlib.nullcontext(None))
    with session_cm as session:
        engine = DenoiseEngine(cfg, grid, dev, cp=cp, impl="fused" if dev.type == "cuda" else "torch",
                               text_cfg=tcfg if a.text_stage else None, mode="serve", profile_dir=a.profile_dir,
                               session=session)
        control = ControlPlane(timeout_seconds=a.control_timeout)
        if a.once:  # one request through the engine, no HTTP (smoke / tests)
            return engine.run({"steps": 2, "seed": 1})
        if control.rank != 0:
            follower_loop(engine, control)
            return None
        import uvicorn

        loop = Rank0Loop(engine, control)
        stop = threading.Event()
        server = uvicorn.Server(uvicorn.Config(make_app(loop.submit), host=a.host, port=a.port, log_level="info"))
        threading.Thread(target=server.run, daemon=True).start()
        try:
            loop.serve_forever(stop)
        except KeyboardInterrupt:
            stop.set()
        return None


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)

    def common(p):
        p.add_argument("--profile-dir", required=True)
        p.add_argument("--layers", type=int, default=48)
        p.add_argument("--no-text-stage", dest="text_stage", action="store_false",
                       help="random context instead of the text encoder stage")
        p.add_argument("--tiny", action="store_true", help="small shapes (smoke runs, CPU)")
        p.add_argument("--cpu", action="store_true")

    common(sub.add_parser("profile", help="profile every stage and save one profile per manager"))
    s = sub.add_parser("serve", help="serve HTTP from the saved profiles")
    common(s)
    s.add_argument("--host", default="127.0.0.1")
    s.add_argument("--port", type=int, default=8000)
    s.add_argument("--shm-namespace", default=None, help="share one host copy of the weights across replicas")
    s.add_argument("--shm-wait-timeout", type=float, default=600.0)
    s.add_argument("--control-timeout", type=float, default=600.0)
    s.add_argument("--once", action="store_true", help="run one request without HTTP and exit")
    return ap.parse_args(argv)


def main(argv=None):
    a = parse_args(argv)
    if a.cmd == "profile":
        for d in cmd_profile(a):
            print(f"saved profile: {d}")
        return None
    return cmd_serve(a)


if __name__ == "__main__":
    _res = main()
    if _res is not None and int(os.environ.get("RANK", "0")) == 0:
        import json

        print(json.dumps(_res))
