"""NUMA interleave of the shared host weight store (no numactl): segment policy at creation,
strict / auto / off modes, and the process-policy launcher."""

import os
import subprocess
import sys
import uuid

import pytest

from flextensor_b200.shm import numa
from flextensor_b200.shm.segment import ShmSegment


def _supported() -> bool:
    try:
        numa.process_policy()
        return True
    except (numa.NumaUnavailable, OSError):
        return False


needs_numa = pytest.mark.skipif(not _supported(), reason="NUMA policy syscalls unavailable here")


def test_parse_node_lists():
    assert numa._parse_list("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert numa._parse_list("0") == [0]
    assert numa.allowed_nodes()  # at least one node


@needs_numa
def test_created_segment_is_interleaved(monkeypatch):
    monkeypatch.setenv("FT_SHM_NUMA_INTERLEAVE", "1")
    seg = ShmSegment.create(f"ftnuma{uuid.uuid4().hex[:8]}", 1 << 21)
    try:
        assert seg.numa_interleaved
        mode, nodes = numa.range_policy(seg.tensor().data_ptr())
        assert mode == numa.MPOL_INTERLEAVE
        assert nodes == numa.allowed_nodes()
        seg.tensor()[:] = 7  # first touch after the policy: pages come from the interleave set
        att = ShmSegment.attach(seg.name)
        assert not att.numa_interleaved and int(att.tensor()[123]) == 7
        att.close()
    finally:
        seg.close()
        seg.unlink()


@needs_numa
def test_off_leaves_the_default_policy(monkeypatch):
    monkeypatch.delenv("FT_SHM_NUMA_INTERLEAVE", raising=False)
    seg = ShmSegment.create(f"ftnuma{uuid.uuid4().hex[:8]}", 1 << 20)
    try:
        assert not seg.numa_interleaved
        assert numa.range_policy(seg.tensor().data_ptr())[0] == numa.MPOL_DEFAULT
    finally:
        seg.close()
        seg.unlink()


def test_strict_raises_auto_warns(monkeypatch, caplog):
    def refuse(addr, length, nodes=None):
        raise numa.NumaUnavailable(1, "refused for the test")

    monkeypatch.setattr(numa, "interleave_range", refuse)
    with pytest.raises(numa.NumaUnavailable):
        numa.apply_to_new_mapping(4096, 4096, mode="on")
    assert numa.apply_to_new_mapping(4096, 4096, mode="auto") is False
    assert "skipped" in caplog.text
    assert numa.apply_to_new_mapping(4096, 4096, mode="off") is False


def test_mode_parsing(monkeypatch):
    for v, want in [("0", "off"), ("", "off"), ("1", "on"), ("auto", "auto"), ("true", "on")]:
        monkeypatch.setenv("FT_SHM_NUMA_INTERLEAVE", v)
        assert numa.interleave_mode() == want
    monkeypatch.setenv("FT_SHM_NUMA_INTERLEAVE", "sometimes")
    with pytest.raises(ValueError):
        numa.interleave_mode()


@needs_numa
def test_exec_launcher_sets_the_process_policy():
    code = "from flextensor_b200.shm import numa; print(numa.process_policy()[0])"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "flextensor_b200.shm.numa", "exec", "--", sys.executable, "-c", code],
                       cwd=root, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert int(r.stdout.strip().splitlines()[-1]) == numa.MPOL_INTERLEAVE
