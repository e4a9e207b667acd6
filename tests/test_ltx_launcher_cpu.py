"""Shell contract of ``examples/ltx_serving/replicas.sh``: with stub ``python`` and ``nginx``
executables first on PATH (they record their arguments and CUDA_VISIBLE_DEVICES, then exit), the
launcher starts one replica per GPU group on consecutive ports, all on one shared-memory
namespace, under torchrun when a replica spans several GPUs, then nginx; with NUMA_INTERLEAVE=1 it
probes the policy first and wraps every replica in the interleave launcher, and a refused probe
stops it before any replica starts."""

import os
import shutil
import stat
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRIPT = os.path.join(ROOT, "examples", "ltx_serving", "replicas.sh")

STUB = """#!/usr/bin/env bash
echo "$(basename "$0") CVD=${CUDA_VISIBLE_DEVICES:-} NUMA=${FT_SHM_NUMA_INTERLEAVE:-} ARGS=$*" >> "$STUB_LOG"
if [ "$(basename "$0")" = python ] && [ "$*" = "-m flextensor_b200.shm.numa probe" ]; then
  exit "${PROBE_RC:-0}"
fi
exit 0
"""


def _run(tmp_path, **env):
    if shutil.which("bash") is None:
        pytest.skip("bash not available")
    bindir = tmp_path / "bin"
    bindir.mkdir()
    for name in ("python", "nginx"):
        p = bindir / name
        p.write_text(STUB)
        p.chmod(p.stat().st_mode | stat.S_IXUSR)
    log = tmp_path / "calls.log"
    e = dict(os.environ, PATH=f"{bindir}:{os.environ['PATH']}", STUB_LOG=str(log), PROFILE_DIR="/tmp/prof",
             SHM_NAMESPACE="ns_test", **env)
    r = subprocess.run(["bash", SCRIPT], env=e, capture_output=True, text=True, timeout=60)
    lines = log.read_text().splitlines() if log.exists() else []
    return r, lines


def test_single_gpu_replicas(tmp_path):
    r, lines = _run(tmp_path, REPLICAS="3", CP="1")
    assert r.returncode == 0, r.stderr
    serves = sorted(l for l in lines if "serve.py serve" in l)
    assert len(serves) == 3
    for i in range(3):
        mine = [l for l in serves if f"--port {8000 + i}" in l]
        assert len(mine) == 1
        assert f"CVD={i} " in mine[0] and "--shm-namespace ns_test" in mine[0] and "--profile-dir /tmp/prof" in mine[0]
        assert "torch.distributed.run" not in mine[0]
    assert any(l.startswith("nginx") and "nginx.conf" in l for l in lines)
    assert not any("numa" in l for l in lines)


def test_context_parallel_replicas_use_torchrun(tmp_path):
    r, lines = _run(tmp_path, REPLICAS="2", CP="4")
    assert r.returncode == 0, r.stderr
    serves = [l for l in lines if "serve.py serve" in l]
    assert len(serves) == 2
    for i, gpus in enumerate(("0,1,2,3", "4,5,6,7")):
        mine = [l for l in serves if f"--port {8000 + i}" in l]
        assert len(mine) == 1 and f"CVD={gpus} " in mine[0]
        assert "-m torch.distributed.run" in mine[0] and "--nproc-per-node 4" in mine[0]
        assert f"--master-port {29500 + i}" in mine[0]


def test_numa_interleave_wraps_every_replica(tmp_path):
    r, lines = _run(tmp_path, REPLICAS="2", CP="1", NUMA_INTERLEAVE="1")
    assert r.returncode == 0, r.stderr
    assert "ARGS=-m flextensor_b200.shm.numa probe" in lines[0]
    serves = [l for l in lines if "serve.py serve" in l]
    assert len(serves) == 2
    for l in serves:
        assert "NUMA=1" in l and "ARGS=-m flextensor_b200.shm.numa exec --" in l


def test_refused_numa_policy_starts_nothing(tmp_path):
    r, lines = _run(tmp_path, REPLICAS="2", CP="1", NUMA_INTERLEAVE="1", PROBE_RC="1")
    assert r.returncode != 0 and "refused" in r.stderr
    assert not any("serve.py" in l for l in lines) and not any(l.startswith("nginx") for l in lines)


def test_profile_dir_is_required(tmp_path):
    if shutil.which("bash") is None:
        pytest.skip("bash not available")
    e = {k: v for k, v in os.environ.items() if k != "PROFILE_DIR"}
    r = subprocess.run(["bash", SCRIPT], env=e, capture_output=True, text=True, timeout=30)
    assert r.returncode != 0 and "PROFILE_DIR" in r.stderr
