"""Model placement snapshots and capacity-safe transition planning.

Used to adopt a saved offload plan into a model that is already loaded (e.g. by vLLM) without
a discovery/profiling cycle: capture where every storage lives now, derive where the plan wants
it, and order the host<->GPU copies so that neither the host nor the GPU ever exceeds what is
free. Nothing here moves memory; :func:`execute_transition` does, once a plan exists.

Parity (behaviour, JSON keys and error classes) with the reference's
``src/flextensor/state_transition.py:15-170,411`` (data model, ``plan_state_transition``),
``model_state_capture.py:55`` (``capture_model_state``) and ``state_adoption.py:159``
(``target_from_profile``). The ordering search is this module's own: a largest-first greedy
that relieves whichever side is short, with an exhaustive memoised search over remaining
sets as the fallback (bounded at ``SEARCH_STATE_LIMIT`` states).
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Literal

import torch

from flextensor_b200.core.host_store import packed_layout

SCHEMA_VERSION = 1
SEARCH_STATE_LIMIT = 10_000
PinningMode = Literal["none", "copy", "in_place"]


# ============================================================================ data model
@dataclass(frozen=True, slots=True)
class TensorState:
    id: str
    names: tuple[str, ...]
    storage_id: str
    logical_bytes: int
    kind: str  # "parameter" | "buffer" | "tensor" (reachable, unregistered)


@dataclass(frozen=True, slots=True)
class StorageState:
    id: str
    device: str  # "cpu" or "cuda:<n>"
    nbytes: int
    pinned: bool


@dataclass(frozen=True, slots=True)
class ModelPlacementState:
    tensors: tuple[TensorState, ...]
    storages: tuple[StorageState, ...]
    schema_version: int = SCHEMA_VERSION

    def to_dict(self) -> dict[str, Any]:
        return {
            "version": self.schema_version,
            "tensors": [{"id": t.id, "names": list(t.names), "storage_id": t.storage_id,
                         "logical_bytes": t.logical_bytes, "kind": t.kind} for t in self.tensors],
            "storages": [{"id": s.id, "device": s.device, "nbytes": s.nbytes, "pinned": s.pinned}
                         for s in self.storages],
        }

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "ModelPlacementState":
        if not isinstance(data, dict):
            raise ValueError("a saved placement must be a JSON object")
        if data.get("version") != SCHEMA_VERSION:
            raise ValueError(f"Unsupported model placement schema version {data.get('version')!r}; "
                             f"expected {SCHEMA_VERSION}")
        trows, srows = data.get("tensors"), data.get("storages")
        if not isinstance(trows, list) or not isinstance(srows, list):
            raise ValueError("placement 'tensors' and 'storages' must both be lists")
        if any(not isinstance(r, dict) or not isinstance(r.get("names"), list) for r in trows):
            raise ValueError("every tensor record needs to be an object carrying a 'names' list")
        if any(not isinstance(r, dict) for r in srows):
            raise ValueError("every storage record needs to be an object")
        try:
            tensors = tuple(TensorState(r["id"], tuple(r["names"]), r["storage_id"], r["logical_bytes"], r["kind"])
                            for r in trows)
            storages = tuple(StorageState(r["id"], r["device"], r["nbytes"], r["pinned"]) for r in srows)
        except (KeyError, TypeError) as e:
            raise ValueError(f"malformed placement record: {e}") from e
        st = cls(tensors=tensors, storages=storages)
        validate_state(st)
        return st


@dataclass(frozen=True, slots=True)
class HostAllocation:
    nbytes: int
    temporary_copy_bytes: int = 0


@dataclass(frozen=True, slots=True)
class TransitionSpec:
    """Memory the loader needs beyond the model's own storages once placement is done."""

    extra_gpu_bytes: int = 0
    pinning_copy_storage_ids: tuple[str, ...] = ()
    host_allocations: tuple[HostAllocation, ...] = ()
    release_host_storage_ids: tuple[str, ...] = ()


@dataclass(frozen=True, slots=True)
class MemoryCapacity:
    host_bytes: int
    gpu_bytes: int


@dataclass(frozen=True, slots=True)
class StorageMigration:
    storage_id: str
    names: tuple[str, ...]
    source_device: str
    destination_device: str
    nbytes: int

    @property
    def to_gpu(self) -> bool:
        return self.destination_device.startswith("cuda:")


@dataclass(frozen=True, slots=True)
class StateTransitionPlan:
    migrations: tuple[StorageMigration, ...]
    pinning_groups: tuple[tuple[str, ...], ...]
    peak_host_bytes: int
    peak_gpu_bytes: int


# ============================================================================ validation
def _nonneg_int(v: object) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


def _check_device(d: object) -> None:
    ok = d == "cpu" or (isinstance(d, str) and d.startswith("cuda:") and d[5:].isdigit())
    if not ok:
        raise ValueError(f"device {d!r} is neither 'cpu' nor a CUDA device with an index")


def validate_state(st: ModelPlacementState) -> None:
    if st.schema_version != SCHEMA_VERSION:
        raise ValueError(f"Unsupported model placement schema version {st.schema_version!r}; "
                         f"expected {SCHEMA_VERSION}")
    seen_ids: set[str] = set()
    seen_names: set[str] = set()
    used: set[str] = set()
    for t in st.tensors:
        if not isinstance(t.id, str) or not t.id or t.id in seen_ids:
            raise ValueError(f"tensor id {t.id!r} is empty or repeated")
        seen_ids.add(t.id)
        if not isinstance(t.names, tuple) or any(not isinstance(n, str) or not n for n in t.names):
            raise ValueError(f"tensor {t.id!r} lists an empty or non-string name")
        dup = seen_names.intersection(t.names)
        if dup or len(set(t.names)) != len(t.names):
            raise ValueError(f"a tensor name appears more than once: {sorted(dup or set(t.names))}")
        seen_names.update(t.names)
        if not isinstance(t.storage_id, str) or not t.storage_id:
            raise ValueError(f"tensor {t.id!r} points at no valid storage")
        used.add(t.storage_id)
        if not _nonneg_int(t.logical_bytes):
            raise ValueError(f"tensor {t.id!r}: logical_bytes has to be an int >= 0")
        if not isinstance(t.kind, str) or not t.kind:
            raise ValueError(f"tensor {t.id!r}: kind is missing")
    sids: set[str] = set()
    for s in st.storages:
        if not isinstance(s.id, str) or not s.id or s.id in sids:
            raise ValueError(f"storage id {s.id!r} is empty or repeated")
        sids.add(s.id)
        _check_device(s.device)
        if not _nonneg_int(s.nbytes):
            raise ValueError(f"storage {s.id!r}: nbytes has to be an int >= 0")
        if type(s.pinned) is not bool:
            raise ValueError(f"storage {s.id!r}: pinned has to be true or false")
        if s.pinned and s.device != "cpu":
            raise ValueError(f"storage {s.id!r} is on {s.device}, which cannot be pinned")
    if used != sids:
        raise ValueError(f"storages and tensor references do not exactly match: missing={sorted(used - sids)}, "
                         f"unreferenced={sorted(sids - used)}")


def _check_transition(cur: ModelPlacementState, tgt: ModelPlacementState, spec: TransitionSpec,
                      cap: MemoryCapacity) -> tuple[dict[str, StorageState], dict[str, StorageState]]:
    validate_state(cur)
    validate_state(tgt)
    if {t.id: t for t in cur.tensors} != {t.id: t for t in tgt.tensors}:
        raise ValueError("the two states hold different tensors; a transition may only move storages")
    cs, ts = {s.id: s for s in cur.storages}, {s.id: s for s in tgt.storages}
    if cs.keys() != ts.keys():
        raise ValueError("the two states hold different storages")
    for sid, c in cs.items():
        t = ts[sid]
        if c.nbytes != t.nbytes:
            raise ValueError(f"storage {sid!r} changes size between the two states")
        if c.pinned and c.device == t.device and not t.pinned:
            raise ValueError(f"storage {sid!r} would lose its pinning, which transitions never do")
        if c.device != t.device and c.device.startswith("cuda:") and t.device.startswith("cuda:"):
            raise ValueError(f"Cross-device CUDA migration is not modeled by this planner: {c.device} -> {t.device}")
    gpus = {s.device for st in (cur, tgt) for s in st.storages if s.device != "cpu"}
    if len(gpus) > 1:
        raise ValueError(f"the capacity check covers one CUDA device, these states use {sorted(gpus)}")
    counts = [cap.host_bytes, cap.gpu_bytes, spec.extra_gpu_bytes]
    counts += [a.nbytes for a in spec.host_allocations] + [a.temporary_copy_bytes for a in spec.host_allocations]
    if not all(_nonneg_int(v) for v in counts):
        raise ValueError("capacities and byte counts have to be ints >= 0")
    pin_ids = set(spec.pinning_copy_storage_ids)
    if len(pin_ids) != len(spec.pinning_copy_storage_ids):
        raise ValueError("pinning_copy_storage_ids repeats an id")
    newly_pinned = {sid for sid, c in cs.items() if not c.pinned and ts[sid].pinned}
    if not pin_ids <= newly_pinned:
        raise ValueError("pinning_copy_storage_ids may only name storages the target state newly pins")
    rel = set(spec.release_host_storage_ids)
    if len(rel) != len(spec.release_host_storage_ids) or not rel <= ts.keys():
        raise ValueError("release_host_storage_ids repeats an id or names an unknown storage")
    if any(ts[sid].device != "cpu" for sid in rel):
        raise ValueError("only host storages of the target state can be released while the loader is built")
    return cs, ts


# ============================================================================ ordering
def _capacity_error(host: int, gpu: int, cap: MemoryCapacity) -> RuntimeError:
    return RuntimeError(f"Insufficient capacity for state transition: host(required={max(0, host)}, "
                        f"available={cap.host_bytes}); gpu(required={max(0, gpu)}, available={cap.gpu_bytes})")


def _delta(m: StorageMigration) -> tuple[int, int]:
    """(host delta, gpu delta) of one migration: the source copy is freed once it has moved."""
    return (-m.nbytes, m.nbytes) if m.to_gpu else (m.nbytes, -m.nbytes)


def _exhaustive_order(ms: tuple[StorageMigration, ...], cap: MemoryCapacity,
                      extra_gpu: int) -> list[StorageMigration] | None:
    """Depth-first over remaining-sets (the running deltas depend only on which moves are done)."""
    full = (1 << len(ms)) - 1
    seen = {full}
    stack: list[tuple[int, int, int, tuple[int, ...]]] = [(full, 0, 0, ())]
    while stack:
        left, h, g, order = stack.pop()
        if left == 0:
            if g + extra_gpu <= cap.gpu_bytes:
                return [ms[i] for i in order]
            continue
        if len(seen) >= SEARCH_STATE_LIMIT:
            raise RuntimeError(f"no capacity-safe move order found within {SEARCH_STATE_LIMIT} search states")
        for i, m in enumerate(ms):
            bit = 1 << i
            if not left & bit:
                continue
            dh, dg = _delta(m)
            nh, ng = h + dh, g + dg
            rest = left ^ bit
            if nh > cap.host_bytes or ng > cap.gpu_bytes or rest in seen:
                continue
            seen.add(rest)
            stack.append((rest, nh, ng, (*order, i)))
    return None


def _order(ms: tuple[StorageMigration, ...], spec: TransitionSpec, cap: MemoryCapacity) -> list[StorageMigration]:
    pending = sorted(ms, key=lambda m: (-m.nbytes, m.names))
    out: list[StorageMigration] = []
    h = g = 0
    while pending:
        fit_up = [m for m in pending if m.to_gpu and g + m.nbytes <= cap.gpu_bytes]
        fit_down = [m for m in pending if not m.to_gpu and h + m.nbytes <= cap.host_bytes]
        if not fit_up and not fit_down:
            alt = _exhaustive_order(ms, cap, spec.extra_gpu_bytes)
            if alt is not None:
                return alt
            final_h = sum(_delta(m)[0] for m in ms)
            raise _capacity_error(final_h, -final_h + spec.extra_gpu_bytes, cap)
        gpu_short = g + sum(m.nbytes for m in pending if m.to_gpu) + spec.extra_gpu_bytes > cap.gpu_bytes
        host_short = h + sum(m.nbytes for m in pending if not m.to_gpu) > cap.host_bytes
        if gpu_short and fit_down:
            pick = fit_down[0]       # free GPU memory first
        elif host_short and fit_up:
            pick = fit_up[0]         # free host memory first
        else:
            pick = (fit_up or fit_down)[0]
        pending.remove(pick)
        out.append(pick)
        dh, dg = _delta(pick)
        h, g = h + dh, g + dg
    return out


def plan_state_transition(current: ModelPlacementState, target: ModelPlacementState, *,
                          transition: TransitionSpec, capacity: MemoryCapacity) -> StateTransitionPlan:
    """Order the storage copies of ``current -> target`` within ``capacity`` (bytes above now)."""
    cs, ts = _check_transition(current, target, transition, capacity)
    names = _names_by_storage(current)
    ms = tuple(StorageMigration(s.id, names[s.id], s.device, ts[s.id].device, s.nbytes)
               for s in current.storages if s.device != ts[s.id].device)
    ordered = _order(ms, transition, capacity)
    h = g = ph = pg = 0
    for m in ordered:
        dh, dg = _delta(m)
        h, g = h + dh, g + dg
        ph, pg = max(ph, h), max(pg, g)
    g += transition.extra_gpu_bytes  # loader slots after placement
    pg = max(pg, g)
    if g > capacity.gpu_bytes:
        raise _capacity_error(h, g, capacity)
    for sid in transition.pinning_copy_storage_ids:
        ph = max(ph, h + ts[sid].nbytes)
    for a in transition.host_allocations:
        h += a.nbytes
        ph = max(ph, h + a.temporary_copy_bytes)
    h -= sum(ts[sid].nbytes for sid in transition.release_host_storage_ids)
    if ph > capacity.host_bytes or h > capacity.host_bytes:
        raise _capacity_error(max(ph, h), g, capacity)
    newly = {sid for sid, c in cs.items() if not c.pinned and ts[sid].pinned}
    groups = tuple(sorted(names[sid] for sid in newly))
    return StateTransitionPlan(tuple(ordered), groups, ph, pg)


def _names_by_storage(st: ModelPlacementState) -> dict[str, tuple[str, ...]]:
    acc: dict[str, list[str]] = {s.id: [] for s in st.storages}
    for t in st.tensors:
        acc[t.storage_id].extend(t.names)
    return {k: tuple(sorted(v)) for k, v in acc.items()}


# ============================================================================ capture
def _reachable_tensors(model: torch.nn.Module) -> dict[int, torch.Tensor]:
    """Tensors held as plain attributes of modules (not registered params/buffers)."""
    out: dict[int, torch.Tensor] = {}
    for m in model.modules():
        for k, v in vars(m).items():
            if k in ("_parameters", "_buffers", "_modules"):
                continue
            if isinstance(v, torch.Tensor) and not isinstance(v, torch.nn.Parameter):
                out.setdefault(id(v), v)
    return out


def _storage_key(name: str, t: torch.Tensor) -> tuple[str, int, int, bool]:
    if t.is_meta:
        raise ValueError(f"{name} is a meta tensor: nothing to capture")
    if t.device.type not in ("cpu", "cuda"):
        raise ValueError(f"Cannot capture tensor {name} on unsupported device {t.device}")
    if t.layout != torch.strided:
        raise ValueError(f"Cannot capture tensor {name} with unsupported layout {t.layout}; "
                         "only torch.strided is supported")
    try:
        st = t.untyped_storage()
    except (NotImplementedError, RuntimeError) as e:
        raise ValueError(f"the storage behind {name} cannot be read") from e
    dev = f"cuda:{t.device.index if t.device.index is not None else torch.cuda.current_device()}" \
        if t.device.type == "cuda" else "cpu"
    return dev, st._cdata, st.nbytes(), bool(t.device.type == "cpu" and t.is_pinned())  # noqa: SLF001


def capture_model_state(model: torch.nn.Module) -> ModelPlacementState:
    """Snapshot tensor identity, aliases and storage placement of ``model`` (no mutation)."""
    if not isinstance(model, torch.nn.Module):
        raise TypeError(f"model must be nn.Module, got {type(model)}")
    found: dict[int, list] = {}  # id(tensor) -> [tensor, names, kind]
    for kind, it in (("parameter", model.named_parameters(remove_duplicate=False)),
                     ("buffer", model.named_buffers(remove_duplicate=False))):
        for n, t in it:
            e = found.get(id(t))
            if e is None:
                found[id(t)] = [t, [n], kind]
            else:
                e[1].append(n)
                if kind == "buffer":
                    e[2] = "buffer"  # buffers stay on the GPU: that classification wins
    for tid, t in _reachable_tensors(model).items():
        found.setdefault(tid, [t, [], "tensor"])
    storages: dict[tuple[str, int], StorageState] = {}
    tensors = []
    for i, (t, ns, kind) in enumerate(found.values()):
        label = ns[0] if ns else f"<reachable:{i}>"
        dev, sid, nbytes, pinned = _storage_key(label, t)
        key = (dev, sid)
        if key not in storages:
            storages[key] = StorageState(f"storage:{dev}:{sid}", dev, nbytes, pinned)
        tensors.append(TensorState(f"tensor:{i}", tuple(sorted(ns)), storages[key].id,
                                   t.numel() * t.element_size(), kind))
    return ModelPlacementState(tuple(tensors), tuple(storages.values()))


# ============================================================================ target from a saved plan
def target_from_profile(current: ModelPlacementState, profile, *, target_device: str, pinning: PinningMode,
                        use_shm: bool) -> tuple[ModelPlacementState, TransitionSpec]:
    """Translate a saved ``TensorManagerState`` into a target placement plus loader needs."""
    profile.validate_internal()
    if not (isinstance(target_device, str) and target_device.startswith("cuda:") and target_device[5:].isdigit()):
        raise ValueError(f"target_device must be an explicit CUDA device, got {target_device!r}")
    cur_gpus = {s.device for s in current.storages if s.device.startswith("cuda:")}
    if cur_gpus - {target_device}:
        raise ValueError(f"Cross-device CUDA migration is not modeled by this planner: "
                         f"{sorted(cur_gpus)} -> {target_device}")
    if pinning not in ("none", "copy", "in_place"):
        raise ValueError(f"Unknown pinning mode {pinning!r}")

    saved = set(profile.tensor_id_to_name_map.values())
    by_name = {n: t for t in current.tensors for n in t.names}
    missing = sorted(saved - by_name.keys())
    unexpected = sorted(t.names for t in current.tensors if t.names and saved.isdisjoint(t.names))
    if missing or unexpected:
        raise ValueError(f"State inventory mismatch: missing_from_model={missing}, unexpected_in_model={unexpected}")
    logical = {n: by_name[n].logical_bytes for n in saved}
    all_stats = [s for v in profile.load_strategy.values() for s in v]
    all_stats += [s for v in profile.release_strategy.values() for s in v]
    all_stats += [s for layer in profile.stats for s in layer.tensors]
    for s in all_stats:
        if s.size_bytes != logical[s.name]:
            raise ValueError(f"TensorStatistics.size_bytes drift for {s.name}: saved={s.size_bytes}, "
                             f"current_logical={logical[s.name]}")
    managed = {s.name for v in profile.load_strategy.values() for s in v} | set(profile.view_tensors_names)
    bad = sorted(n for n in managed if by_name[n].kind == "buffer")
    if bad:
        raise ValueError(f"Registered buffer(s) must remain final-GPU, not managed: {bad}")

    strategy_loader = profile.loader_type == "strategy"
    dest: dict[str, set[str]] = {s.id: set() for s in current.storages}
    for t in current.tensors:
        hit = saved.intersection(t.names)
        if hit:
            dest[t.storage_id].add("cpu" if hit & managed else target_device)
    for d in dest.values():
        if not d:
            d.add(target_device)
    clash = sorted(k for k, d in dest.items() if len(d) != 1)
    if clash:
        raise ValueError(f"Contradictory alias destinations for shared storage: {clash}")
    managed_sids = {k for k, d in dest.items() if next(iter(d)) == "cpu"}
    tgt_storages = []
    for s in current.storages:
        dev = next(iter(dest[s.id]))
        pinned = (s.pinned or (strategy_loader and pinning != "none")) if dev == "cpu" else False
        tgt_storages.append(replace(s, device=dev, pinned=pinned))
    target = ModelPlacementState(current.tensors, tuple(tgt_storages))

    if strategy_loader:
        extra = _strategy_peak_gpu_bytes(profile, logical, managed)
        allocs: tuple[HostAllocation, ...] = ()
        release: tuple[str, ...] = ()
    elif profile.loader_type in ("allocation_block_transfer", "raw_block_transfer"):
        views: dict[str, list[tuple[str, ...]]] = {}
        for t in current.tensors:
            if t.storage_id in managed_sids:
                views.setdefault(t.storage_id, []).append(t.names)
        shared = {k: v for k, v in views.items() if len(v) > 1}
        if shared:
            raise ValueError(f"Block loaders cannot preserve distinct tensor views sharing storage: {shared}")
        load = {k: v for k, v in profile.load_strategy.items() if v}
        if use_shm and profile.shm_block_name_map is not None and set(profile.shm_block_name_map) != set(load):
            raise ValueError("Saved state mismatch: shm_block_name_map must cover exactly the nonempty load labels. "
                             "Re-profile the model.")
        if profile.loader_type == "raw_block_transfer":
            extra = sum(profile.block_sizes.values())
            label_bytes = dict(profile.label_to_size_map)
            labels = list(load)
            follower = False
        else:
            label_bytes = {k: packed_layout([logical[n] for n in dict.fromkeys(s.name for s in v)])[1]
                           for k, v in load.items()}
            extra = sum(max(label_bytes[l] for l in ls) for ls in profile.allocation_ordered.values() if ls)
            labels = [l for ls in profile.allocation_ordered.values() for l in ls]
            follower = use_shm and profile.shm_block_name_map is not None
        copy_blocks = pinning == "copy" and not (profile.loader_type == "allocation_block_transfer" and use_shm)
        allocs = () if follower else tuple(
            HostAllocation(label_bytes[l], label_bytes[l] if copy_blocks else 0) for l in labels)
        release = tuple(s.id for s in current.storages if s.id in managed_sids)
    else:
        raise ValueError(f"Unknown loader type: {profile.loader_type}")
    tmap = {s.id: s for s in target.storages}
    pin_copy = tuple(s.id for s in current.storages if pinning == "copy" and not s.pinned and tmap[s.id].pinned)
    return target, TransitionSpec(extra, pin_copy, allocs, release)


def _strategy_peak_gpu_bytes(profile, logical: dict[str, int], managed: set[str]) -> int:
    """Peak bytes of managed tensors on the GPU over one pass of a per-tensor (strategy) plan."""
    scheduled: set[str] = set()
    in_layers: set[str] = set()
    preloaded: set[str] = set()
    for layer in profile.stats:
        scheduled.update(s.name for s in profile.load_strategy.get(layer.label, ()))
        names = {s.name for s in layer.tensors}
        in_layers |= names
        preloaded |= names - scheduled
    live = (preloaded | (managed - in_layers)) & managed
    cur = sum(logical[n] for n in live)
    peak = cur
    for layer in profile.stats:
        for s in profile.load_strategy.get(layer.label, ()):
            if s.name not in live:
                live.add(s.name)
                cur += logical[s.name]
        peak = max(peak, cur)
        for s in profile.release_strategy.get(layer.label, ()):
            if s.name in live:
                live.remove(s.name)
                cur -= logical[s.name]
    return peak


# ============================================================================ execution
def execute_transition(model: torch.nn.Module, plan: StateTransitionPlan, *, pin=None) -> None:
    """Move storages in plan order (not transactional: completed moves are kept on error).

    Every tensor sharing a storage is re-pointed at the moved copy, so aliases stay aliases.
    ``pin(t) -> t`` page-locks host copies (the manager's pinner); CUDA graphs or compiled
    graphs captured before this call hold stale pointers afterwards.
    """
    live: dict[str, list[tuple[str, torch.Tensor]]] = {}
    for kind, it in (("parameter", model.named_parameters(remove_duplicate=False)),
                     ("buffer", model.named_buffers(remove_duplicate=False))):
        for n, t in it:
            dev, sid, _, _ = _storage_key(n, t)
            live.setdefault(f"storage:{dev}:{sid}", []).append((n, t))
    done: list[str] = []
    pinned_names = {n for g in plan.pinning_groups for n in g}
    for m in plan.migrations:
        try:
            group = live.get(m.storage_id, [])
            if not group:
                continue
            moved: dict[int, torch.Tensor] = {}
            for n, t in group:
                if id(t) in moved:
                    continue
                dst = torch.device(m.destination_device)
                nt = t.data.to(dst, non_blocking=False)
                if dst.type == "cpu" and pin is not None and (n in pinned_names or m.destination_device == "cpu"):
                    nt = pin(nt)
                t.data = nt
                moved[id(t)] = nt
            done.append(m.storage_id)
        except Exception as e:
            raise RuntimeError(f"state adoption failed at storage {m.storage_id} ({', '.join(m.names[:3])}); "
                               f"completed={done}") from e
