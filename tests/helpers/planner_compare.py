"""Subprocess body of the planner fidelity test: runs the reference planner (installed under
baseline/_ref) and ours on the same synthetic profiles and scores both plans with the
reference's own evaluator (neutral judge). Prints one JSON line per case."""

import json
import os
import random
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def profiles():
    rng = random.Random(0)
    out = []
    # Wan-like: 40 equal blocks of 0.70 GB, 38 ms each; transfers at ~45 GB/s
    out.append(("wan40", [(38.0, [700_000_000 // 4] * 4) for _ in range(40)]))
    # uneven random profiles
    for k in range(4):
        n = rng.randint(6, 24)
        out.append((f"rand{k}", [(rng.uniform(1.0, 30.0), [rng.randint(8, 200) << 20 for _ in range(rng.randint(1, 4))])
                                 for _ in range(n)]))
    return out


def build(LS, TS, spec):
    stats, tid = [], 0
    for i, (dur, sizes) in enumerate(spec):
        ts = []
        for s in sizes:
            ts.append(TS(tensor_id=tid, name=f"l{i}.t{tid}", size_bytes=s, load_time_ms=s / 45e6))
            tid += 1
        stats.append(LS(label=f"l{i}", tensors=ts, duration=dur))
    return stats


def main():
    sys.path.insert(0, os.path.join(ROOT, "baseline", "shims"))
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    os.environ.setdefault("DISABLE_BEARTYPE", "1")
    from flextensor.collectors import LayerStatistics as RLS, TensorStatistics as RTS
    from flextensor.memory_transfer_interpolator import MemoryTransferInterpolator as RInterp
    from flextensor.strategy.adaptive import AdaptiveStrategy as RAdaptive
    from flextensor.strategy.evaluation import evaluate_strategy_result as r_eval

    sys.path.insert(0, ROOT)
    from flextensor_b200.core.stats import LayerStatistics as OLS, TensorStatistics as OTS
    from flextensor_b200.planner import AdaptiveStrategy as OAdaptive

    mem = {1 << 20: 0.03, 1 << 24: 0.4, 1 << 27: 3.0, 1 << 30: 23.0}
    for name, spec in profiles():
        total = sum(sum(s) for _, s in spec)
        for frac in (None, 0.35, 0.6):
            budget = None if frac is None else int(total * frac)
            rstats, ostats = build(RLS, RTS, spec), build(OLS, OTS, spec)
            interp = RInterp(mem)
            row = {"case": name, "budget_frac": frac}
            for who, strat, stats in (("ref", RAdaptive(n_blocks=2, min_blocks=2), rstats),
                                      ("ours", OAdaptive(n_blocks=2, min_blocks=2), ostats)):
                try:
                    res = strat.compute(stats, mem, budget)
                except Exception as e:  # noqa: BLE001
                    row[who] = {"error": f"{type(e).__name__}: {e}"[:200]}
                    continue
                # score with the reference evaluator on the reference's stat objects
                smap = {k: [RTS(**t.model_dump()) for t in v] for k, v in res.strategy_map.items()}
                rres = type("R", (), {"strategy_map": smap, "block_data": res.block_data})
                try:
                    sc = r_eval(rres, rstats, who, interp, budget)
                    row[who] = {"peak": sc.peak_memory_bytes, "overhead": round(sc.estimated_overhead, 5), "valid": sc.is_valid}
                except Exception as e:  # noqa: BLE001
                    row[who] = {"error": f"eval {type(e).__name__}: {e}"[:200]}
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
