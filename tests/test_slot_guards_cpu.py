"""Debug guards around ring slots (``FT_DEBUG_CANARY=1``): a write that runs past a slot into its
guard region is reported after the forward with the slot's id; clean passes report nothing.
Also: the NVTX switch only adds host-side ranges (the loader works with it on). CPU device."""

import torch

from flextensor_b200.core.host_store import pack_tensors
from flextensor_b200.runtime import loaders as L
from flextensor_b200.runtime.engine import PyTransferEngine


def _loader(monkeypatch, canary=True, nvtx=False):
    monkeypatch.setattr(L, "DEBUG_CANARY", canary)
    monkeypatch.setattr(L, "NVTX", nvtx)
    # the copy issued on entering trap Lk carries the weights of trap Lk+1
    blocks = {f"L{i}": pack_tensors(f"L{i}", [(i, f"w{i}", torch.full((64,), float(i)))], pinned=False)
              for i in range(2)}
    plan = L.SlotPlan(order=["L0", "L1", "L2"], transfer_slot={"L0": 0, "L1": 1},
                      t2c={"L0": "L1", "L1": "L2"}, slot_bytes={0: 256, 1: 256}, host_blocks=blocks)
    return L.BlockLoader(torch.device("cpu"), plan, PyTransferEngine(torch.device("cpu"), 2))


def _forward(ld):
    for c in ("L0", "L1", "L2"):
        ld.enter(c)
        ld.exit(c)


def test_clean_passes_keep_guards(monkeypatch):
    ld = _loader(monkeypatch)
    for _ in range(2):
        _forward(ld)
    assert ld.canary and ld.check_canaries() == []


def test_write_past_a_slot_is_reported(monkeypatch):
    ld = _loader(monkeypatch)
    _forward(ld)
    base = ld.slots[1]
    # one byte past the end of slot 1, inside its trailing guard (same allocation)
    torch.as_strided(base, (1,), (1,), base.storage_offset() + base.numel()).fill_(0)
    try:
        _forward(ld)
    except L.SlotGuardError as e:
        assert "[1]" in str(e)
    else:
        raise AssertionError("guard overwrite not reported")


def test_guards_off_by_default(monkeypatch):
    ld = _loader(monkeypatch, canary=False)
    _forward(ld)
    assert not ld.canary and ld._guards == {}


def test_nvtx_ranges_balanced(monkeypatch):
    ld = _loader(monkeypatch, canary=False, nvtx=True)
    pushes = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: pushes.append(name))
    pops = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: pops.append(1))
    _forward(ld)
    assert len(pushes) == len(pops) and "ft:L1" in pushes and any(p.startswith("ft:h2d:") for p in pushes)
