"""SharedOffloadSession: one host copy of the weights for every local worker.

Flow per manager name (reference: ``src/flextensor/shared_offload.py:110-518``):

1. Every worker builds a session with the same run namespace; each manager
   name maps to an independent child namespace ``ft_<sha256(ns\\0name)[:12]>``.
2. ``offload_from_profile`` runs a creator election (:class:`ShmCoordinator`).
3. Creator: reads ``profile.json``, builds the checkpoint-backed model, offloads
   it with SHM weight blocks (packed + ``cudaHostRegister``-ed), publishes the
   resident tensors (FTTS v1 store) and the live plan, then marks READY. Any
   exception marks FAILED with the message.
4. Follower: waits for READY (bounded by ``wait_timeout``, with creator
   heartbeat liveness), builds the model on ``meta``, materialises resident
   tensors from the store, and attaches to the same SHM weight blocks.

Each process then streams from the shared pinned pages with its own copy
engine; no process ever copies the offloaded weights a second time.
"""

from __future__ import annotations

import math
import os
import re
import threading
from collections.abc import Callable
from typing import Any

import torch
from torch import nn

from flextensor_b200.config import OffloadConfig
from flextensor_b200.core.state import PROFILE_FILENAME, TensorManagerState
from flextensor_b200.runtime.manager import DEFAULT_MANAGER_NAME, get_offload_manager
from flextensor_b200.shm.coordinator import ShmCoordinator, cleanup_namespace, retire_abandoned
from flextensor_b200.shm.namespace import session_namespace
from flextensor_b200.shm.tensor_store import SharedTensorStore

_NS_RE = re.compile(r"[A-Za-z0-9._-]{1,64}")


def _normalize(namespace: Any, wait_timeout: Any) -> tuple[str, float]:
    if not isinstance(namespace, str) or _NS_RE.fullmatch(namespace) is None:
        raise ValueError("namespace must be 1-64 POSIX-safe characters: letters, digits, '.', '_' or '-'")
    try:
        t = float(wait_timeout)
    except (TypeError, ValueError) as exc:
        raise ValueError("wait_timeout must be a number") from exc
    if not math.isfinite(t) or t < 0:
        raise ValueError("wait_timeout must be a non-negative finite number")
    return namespace, t


class SharedOffloadSession:
    def __init__(self, namespace: str, *, wait_timeout: Any = 300.0) -> None:
        self.namespace, self.wait_timeout = _normalize(namespace, wait_timeout)
        self._owner = (os.getpid(), threading.get_ident())
        self._coords: dict[str, ShmCoordinator] = {}
        self._stores: dict[str, SharedTensorStore] = {}
        self._closed = False

    @staticmethod
    def validate_options(namespace: object, *, wait_timeout: Any = 300.0) -> None:
        _normalize(namespace, wait_timeout)

    def _check_owner(self) -> None:
        if (os.getpid(), threading.get_ident()) != self._owner:
            raise RuntimeError("SharedOffloadSession is process- and thread-affine; build one per worker")
        if self._closed:
            raise RuntimeError("SharedOffloadSession is closed")

    def namespace_for(self, name: str) -> str:
        if not isinstance(name, str) or _NS_RE.fullmatch(name) is None:
            raise ValueError("manager name must be 1-64 POSIX-safe characters")
        return session_namespace(self.namespace, name)

    @staticmethod
    def cleanup_namespace(namespace: str, *, manager_names, timeout: Any = 60.0) -> None:
        if isinstance(manager_names, str):
            raise ValueError("manager_names must be an iterable of manager names, not a string")
        names = list(manager_names)
        if not names:
            raise ValueError("manager_names must not be empty")
        s = SharedOffloadSession(namespace)
        for n in dict.fromkeys(names):
            retire_abandoned(s.namespace_for(n))

    def offload_from_profile(self, profile_directory: str | os.PathLike, *, config: OffloadConfig,
                             name: str = DEFAULT_MANAGER_NAME, creator_model_factory: Callable[[], nn.Module],
                             follower_model_factory: Callable[[], nn.Module],
                             materialize_device: torch.device | str | None = None,
                             compile_fn: Callable[[nn.Module], nn.Module] | None = None) -> nn.Module:
        self._check_owner()
        if config.transfer_mode == "strategy":
            raise ValueError("shared offload needs a block transfer_mode")
        ns = self.namespace_for(name)
        cfg = config.model_copy(update={"shm_enabled": True, "shm_namespace": ns,
                                        "shm_wait_timeout": self.wait_timeout})
        coord = ShmCoordinator(ns)
        self._coords[name] = coord
        om = get_offload_manager(name)
        dev = materialize_device or (torch.device("cuda", cfg.gpu_device) if torch.cuda.is_available() else "cpu")
        try:
            if coord.is_creator:
                state = TensorManagerState.load_from_file(os.path.join(os.fspath(profile_directory), PROFILE_FILENAME))
                model = creator_model_factory()
                om.init(cfg)
                om.load_profile(os.fspath(profile_directory))
                model = om.offload(model, cfg, compile_fn=compile_fn)
                tm = om.get_tensor_manager()
                live = tm.export_state()
                resident = [tm.id_to_name[t] for t in sorted(tm.resident)]
                self._stores[name] = SharedTensorStore.create_from_model(ns, model, resident)
                coord.write_profile(TensorManagerState.save_state_to_bytes(live))
                coord.notify_ready()
                _ = state
                return model
            coord.wait_for_ready(self.wait_timeout or None)
            live = coord.read_profile()
            model = follower_model_factory()
            store = SharedTensorStore.attach(ns)
            self._stores[name] = store
            store.materialize_into(model, dev)
            om.init(cfg)
            tm = om.get_tensor_manager()
            tm.load_from_shm = True
            return om.offload_from_state(model, live, cfg)
        except BaseException as exc:
            if coord.is_creator:
                try:
                    coord.mark_failed(f"{type(exc).__name__}: {exc}")
                except Exception:  # noqa: BLE001
                    pass
            raise

    def __enter__(self) -> "SharedOffloadSession":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self, name: str | None = None) -> None:
        names = [name] if name is not None else list(self._coords)
        for n in names:
            st = self._stores.pop(n, None)
            if st is not None:
                st.close()
            try:
                get_offload_manager(n).release()
            finally:
                c = self._coords.pop(n, None)
                if c is not None:
                    c.close()
        if name is None:
            self._closed = True


__all__ = ["SharedOffloadSession", "cleanup_namespace"]
