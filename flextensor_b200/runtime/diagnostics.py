"""Plan diagnostics logged on the ``flextensor_b200.diagnostics`` logger
(block table and per-trap durations; reference ``src/flextensor/strategy/utils.py:309-465``)."""

from __future__ import annotations

import logging

log = logging.getLogger("flextensor_b200.diagnostics")


def plan_table(tm) -> str:
    lines = [f"{'trap':<36} {'ms':>9} {'MB':>9} {'streamed MB':>12} {'slot':>5} -> compute"]
    loader = tm.loader
    slots = getattr(getattr(loader, "plan", None), "transfer_slot", {})
    t2c = getattr(getattr(loader, "plan", None), "t2c", {})
    load = tm.strategy_result.strategy_map if tm.strategy_result is not None else {}
    for l in tm.layer_stats:
        mb = sum(t.size_bytes for t in l.tensors) / 2**20
        smb = sum(t.size_bytes for t in load.get(l.label, ())) / 2**20
        lines.append(f"{l.label[:36]:<36} {l.duration:>9.3f} {mb:>9.1f} {smb:>12.1f} "
                     f"{slots.get(l.label, '-'):>5} -> {t2c.get(l.label, '')}")
    return "\n".join(lines)


def log_plan(tm) -> None:
    log.info("offload plan:\n%s", plan_table(tm))
