"""Plan diagnostics on the ``flextensor_b200.diagnostics`` logger, emitted together when a plan is
built with ``enable_diagnostics`` (the reference logs the same three views: per-trap durations,
the transfer benchmark and the block assignment; ``src/flextensor/tensor_manager.py:1267-1293``,
``strategy/utils.py:309-465``, ``memory_transfer_benchmark.py:26-56``).

* :func:`duration_table` -- per trap: samples, median / mean / spread (profiling collector), or
  the effective durations the plan used;
* :func:`transfer_table` -- the host -> device benchmark: size, time, bandwidth;
* :func:`plan_table` -- per trap: its bytes, what streams into it, the ring slot, the trap whose
  compute the copy overlaps, the copy time the benchmark predicts, the compute window it has and
  the part left exposed; then every slot's size and users, and the plan totals.
"""

from __future__ import annotations

import logging

log = logging.getLogger("flextensor_b200.diagnostics")


def _mb(n: float) -> float:
    return n / 2**20


def duration_table(tm) -> str:
    from flextensor_b200.runtime.profiling_quality import (LayerStatisticsAnalyzer,
                                                           format_effective_layer_duration_table)

    collector = getattr(tm, "collector", None)
    if collector is not None and collector.labels():
        return LayerStatisticsAnalyzer(collector).format_statistics_table()
    return format_effective_layer_duration_table(tm.layer_stats)


def transfer_table(memory_stats: dict[int, float] | None) -> str:
    if not memory_stats:
        return "(no transfer benchmark)"
    rows = [f"{'bytes':>14} {'MiB':>10} {'ms':>10} {'GB/s':>9}"]
    for n, ms in sorted(memory_stats.items()):
        rows.append(f"{n:>14} {_mb(n):>10.2f} {ms:>10.3f} {(n / (ms * 1e6) if ms > 0 else 0.0):>9.2f}")
    return "\n".join(rows)


def _window_ms(order: list[str], durations: dict[str, float], issue: str, need: str) -> float:
    """Compute time from the start of trap ``issue`` up to (not including) trap ``need``, wrapping
    to the next pass when ``need`` comes first."""
    if issue not in order or need not in order:
        return 0.0
    i, j = order.index(issue), order.index(need)
    span = order[i:j] if i < j else order[i:] + order[:j]
    return sum(durations.get(l, 0.0) for l in span)


def plan_rows(tm) -> tuple[list[dict], dict]:
    """The plan table's data: one dict per trap and a totals dict (also used by tests)."""
    plan = getattr(getattr(tm, "loader", None), "plan", None)
    slots = getattr(plan, "transfer_slot", {}) or {}
    t2c = getattr(plan, "t2c", {}) or {}
    blocks = getattr(plan, "host_blocks", {}) or {}
    result = getattr(tm, "strategy_result", None)
    load = result.strategy_map if result is not None else {}
    order = [l.label for l in tm.layer_stats]
    durations = {l.label: float(l.duration) for l in tm.layer_stats}
    interp = None
    if getattr(tm, "memory_stats", None):
        from flextensor_b200.planner.interpolator import create_interpolator_from_benchmarks

        interp = create_interpolator_from_benchmarks(tm.memory_stats)
    rows = []
    for l in tm.layer_stats:
        streamed = sum(t.size_bytes for t in load.get(l.label, ()))
        if l.label in blocks:
            streamed = max(streamed, int(getattr(blocks[l.label], "total", None) or blocks[l.label].nbytes))
        issue = t2c.get(l.label)
        copy_ms = interp.bytes_to_duration(streamed) if (interp is not None and streamed) else 0.0
        window = _window_ms(order, durations, issue, l.label) if issue else 0.0
        rows.append({"label": l.label, "ms": durations[l.label], "bytes": sum(t.size_bytes for t in l.tensors),
                     "streamed": streamed, "slot": slots.get(l.label), "issue": issue, "copy_ms": copy_ms,
                     "window_ms": window, "exposed_ms": max(0.0, copy_ms - window) if streamed else 0.0})
    copy_total = sum(r["copy_ms"] for r in rows)
    exposed = sum(r["exposed_ms"] for r in rows)
    slot_bytes = dict(getattr(plan, "slot_bytes", {}) or {})
    totals = {"compute_ms": sum(durations.values()), "streamed": sum(r["streamed"] for r in rows),
              "resident": int(getattr(tm, "unmapped_bytes", 0) or 0), "slots": sum(slot_bytes.values()),
              "copy_ms": copy_total, "exposed_ms": exposed,
              "hidden_pct": 100.0 * (1.0 - exposed / copy_total) if copy_total > 0 else 100.0,
              "slot_bytes": slot_bytes,
              "slot_users": {s: [t for t, b in slots.items() if b == s] for s in slot_bytes}}
    return rows, totals


def plan_table(tm) -> str:
    rows, tot = plan_rows(tm)
    name = type(getattr(tm, "strategy", None)).__name__
    out = [f"plan ({name}): {len(rows)} traps",
           f"{'trap':<32} {'ms':>8} {'MiB':>8} {'stream MiB':>10} {'slot':>4} {'copied during':<24} "
           f"{'copy ms':>8} {'window ms':>9} {'exposed':>8}"]
    for r in rows:
        slot = "-" if r["slot"] is None else str(r["slot"])
        issue = (r["issue"] or "-")[:24]
        out.append(f"{r['label'][:32]:<32} {r['ms']:>8.3f} {_mb(r['bytes']):>8.1f} {_mb(r['streamed']):>10.1f} "
                   f"{slot:>4} {issue:<24} {r['copy_ms']:>8.3f} {r['window_ms']:>9.3f} {r['exposed_ms']:>8.3f}")
    for s, n in sorted(tot["slot_bytes"].items()):
        users = tot["slot_users"].get(s, [])
        out.append(f"slot {s}: {_mb(n):.1f} MiB, {len(users)} transfers: {', '.join(users[:6])}"
                   f"{' ...' if len(users) > 6 else ''}")
    out.append(f"total: compute {tot['compute_ms']:.2f} ms, streamed {_mb(tot['streamed']):.1f} MiB, "
               f"resident {_mb(tot['resident']):.1f} MiB, slots {_mb(tot['slots']):.1f} MiB, "
               f"copies {tot['copy_ms']:.2f} ms (predicted exposed {tot['exposed_ms']:.2f} ms, "
               f"{tot['hidden_pct']:.1f} % hidden)")
    return "\n".join(out)


def log_plan(tm) -> None:
    """Log the duration, transfer and plan tables (called when a plan is built). A plan built
    from profiling already had its per-trap durations logged by the profiling-quality report;
    a restored plan logs the durations it was planned with."""
    collector = getattr(tm, "collector", None)
    if collector is None or not collector.labels():
        log.info("trap durations:\n%s", duration_table(tm))
    log.info("host -> device transfer benchmark:\n%s", transfer_table(getattr(tm, "memory_stats", None)))
    log.info("offload plan:\n%s", plan_table(tm))
