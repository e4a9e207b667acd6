"""Bounded CPU control plane for multi-rank replicas (context-parallel serving and the like).

Commands and per-request outcomes travel over a Gloo group with a short timeout; the data
plane (NCCL, peer memory) never carries control traffic. Failure handling follows three
rules, the same ones the reference's context-parallel serving uses (``examples/ltx23/outpaint/
context_parallel.py:406-625``):

* a leader broadcast that does not complete within ``timeout`` fires a watchdog that ends the
  process (the stuck collective cannot be cancelled; the launcher then reaps the replica);
* any failed control collective *poisons* the replica: the error is raised as
  :class:`ReplicaFatalError` and every later collective is refused, so no rank enters a
  collective its peers have abandoned;
* a poisoned replica skips ``destroy_process_group`` (which would wait for missing peers).

``terminate`` is injectable so tests can observe the watchdog without ending the test runner.
"""

from __future__ import annotations

import datetime
import logging
import os
import threading
from typing import Any, Callable

LOGGER = logging.getLogger(__name__)


class ReplicaFatalError(RuntimeError):
    """The replica can no longer take part in collectives; the process must exit."""


def _default_terminate(code: int) -> None:
    os._exit(code)


class ControlPlane:
    def __init__(self, timeout_seconds: float = 30.0, group=None, *,
                 terminate: Callable[[int], None] = _default_terminate):
        import torch.distributed as dist

        self.enabled = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
        self.timeout = float(timeout_seconds)
        self._terminate = terminate
        self.poisoned = False
        self.poison_reason: str | None = None
        if not self.enabled:
            self.rank, self.size, self.group = 0, 1, None
            return
        self.rank, self.size = dist.get_rank(), dist.get_world_size()
        if group is None:
            backend = dist.get_backend()
            group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=self.timeout)) \
                if backend != "gloo" else dist.new_group(timeout=datetime.timedelta(seconds=self.timeout))
        self.group = group

    @property
    def is_leader(self) -> bool:
        return self.rank == 0

    # ------------------------------------------------------------------ failure state
    def ensure_usable(self) -> None:
        if self.poisoned:
            raise ReplicaFatalError(f"replica already poisoned: {self.poison_reason}")

    def mark_poisoned(self, reason: str) -> None:
        if not self.poisoned:
            self.poisoned, self.poison_reason = True, reason
            LOGGER.critical("replica no longer usable: %s", reason)

    def fail(self, reason: str, cause: BaseException | None = None):
        self.mark_poisoned(reason)
        raise ReplicaFatalError(reason) from cause

    def terminate(self, reason: str, code: int = 1) -> None:
        self.mark_poisoned(reason)
        self._terminate(code)

    # ------------------------------------------------------------------ collectives
    def broadcast_object(self, value: Any = None, timeout_seconds: float | None = None) -> Any:
        """Leader -> everyone. The leader's send is bounded by a watchdog thread."""
        import torch.distributed as dist

        self.ensure_usable()
        if not self.enabled:
            return value
        done = threading.Event()
        dog = None
        if self.is_leader:
            limit = self.timeout if timeout_seconds is None else float(timeout_seconds)
            if limit <= 0:
                raise ValueError("broadcast timeout must be positive")

            def watch() -> None:
                if not done.wait(limit):
                    LOGGER.critical("command broadcast exceeded %.1fs; terminating the replica", limit)
                    self.terminate(f"broadcast stalled for {limit:.1f}s", code=3)

            dog = threading.Thread(target=watch, name="ft-broadcast-watchdog", daemon=True)
            dog.start()
        box = [value if self.is_leader else None]
        try:
            dist.broadcast_object_list(box, src=0, group=self.group)
        except Exception as e:  # noqa: BLE001 - every failure poisons the replica
            self.fail("command broadcast failed", e)
        finally:
            done.set()
            if dog is not None:
                dog.join(timeout=1)
        return box[0]

    def exchange_status(self, status: dict) -> list:
        """Every rank's outcome of the current request (bounded by the group timeout)."""
        import torch.distributed as dist

        self.ensure_usable()
        if not self.enabled:
            return [status]
        out: list = [None] * self.size
        try:
            dist.all_gather_object(out, status, group=self.group)
        except Exception as e:  # noqa: BLE001
            self.fail(f"request outcome exchange exceeded the {self.timeout:g}s control timeout", e)
        return out

    def request_ok(self, status: dict) -> bool:
        """All ranks succeeded? A failure anywhere poisons every replica member."""
        statuses = self.exchange_status(status)
        bad = [s for s in statuses if not (isinstance(s, dict) and s.get("ok"))]
        if bad:
            self.mark_poisoned(f"{len(bad)} rank(s) failed the request: {bad[:2]}")
            return False
        return True

    def close(self) -> None:
        import torch.distributed as dist

        if self.enabled and not self.poisoned and dist.is_initialized():
            dist.destroy_process_group()
