"""Creator/follower coordination over shared memory (protocol v4).

Wire format kept from the reference (``src/flextensor/shm/coord_block.py:17-141``):
the coordination block ``{ns}_crd`` starts with the header
``!I64sIQII160s`` = (version-string length, version string, protocol version,
creator participant id, state in {INITIALIZING=1, READY=2, FAILED=3},
failure-text length, failure text). The published plan lives in ``{ns}_prof``
as a 4-byte big-endian length + compact JSON (``TensorManagerState``).

Liveness (this package's design): every participant owns one slot in
``{ns}_hb`` -- 64 slots of ``<QQd8x`` (participant id, pid, last-beat unix
time) -- refreshed by a daemon thread every ``lease/4`` seconds. A follower
waiting on INITIALIZING raises :class:`ShmCreatorDiedError` once the creator's
slot is older than the lease, :class:`ShmCreatorFailedError` on FAILED, and
``TimeoutError`` past ``timeout``. Nothing probes PIDs: a lease is the only
liveness signal, which also works across PID namespaces.

Election: whoever creates ``{ns}_crd`` with ``O_EXCL`` under the namespace's
file lock is the creator; everyone else is a follower.
"""

from __future__ import annotations

import logging
import os
import secrets
import struct
import threading
import time
from dataclasses import dataclass
from enum import IntEnum

from flextensor_b200.shm.namespace import (
    SHM_PROTOCOL_VERSION,
    coord_block_name,
    heartbeat_block_name,
    profile_block_name,
)
from flextensor_b200.shm.segment import ProcessFileLock, ShmSegment, shm_exists, shm_unlink

logger = logging.getLogger(__name__)

_VERSION_MAX = 64
_FAILURE_MAX = 160
_HDR = struct.Struct(f"!I{_VERSION_MAX}sIQII{_FAILURE_MAX}s")
COORD_HEADER_SIZE = _HDR.size
_HB_SLOTS = 64
_HB = struct.Struct("<QQd8x")
DEFAULT_LEASE_S = 30.0
POLL_S = 0.25


class ShmCoordinatorError(RuntimeError):
    pass


class ShmCreatorDiedError(ShmCoordinatorError):
    pass


class ShmCreatorFailedError(ShmCoordinatorError):
    pass


class CoordinatorState(IntEnum):
    INITIALIZING = 1
    READY = 2
    FAILED = 3


@dataclass
class CoordBlockHeader:
    flextensor_version: str
    protocol_version: int
    creator_pid: int = 0
    state: CoordinatorState | int = CoordinatorState.INITIALIZING
    failure_message: str = ""

    def write_to(self, buf, offset: int = 0) -> None:
        v = self.flextensor_version.encode()[:_VERSION_MAX]
        f = self.failure_message.encode()[:_FAILURE_MAX].decode("utf-8", errors="ignore").encode()
        _HDR.pack_into(buf, offset, len(v), v.ljust(_VERSION_MAX, b"\0"), self.protocol_version,
                       self.creator_pid, int(self.state), len(f), f.ljust(_FAILURE_MAX, b"\0"))

    @classmethod
    def read_from(cls, buf, offset: int = 0) -> "CoordBlockHeader":
        vl, vb, proto, pid, state, fl, fb = _HDR.unpack_from(buf, offset)
        if vl > _VERSION_MAX or fl > _FAILURE_MAX:
            raise RuntimeError("corrupt coordination header")
        try:
            st = CoordinatorState(state)
        except ValueError:
            st = state
        return cls(vb[:vl].decode(), proto, pid, st, fb[:fl].decode())

    def validate(self, expected_version: str, expected_protocol: int) -> None:
        if self.flextensor_version != expected_version:
            raise RuntimeError(f"version mismatch: SHM created by {self.flextensor_version}, this process is "
                               f"{expected_version}. All processes must use the same version.")
        if self.protocol_version != expected_protocol:
            raise RuntimeError(f"SHM protocol version mismatch: SHM uses protocol {self.protocol_version}, "
                               f"this process expects {expected_protocol}.")
        if self.creator_pid <= 0:
            raise RuntimeError("SHM protocol v3+ requires a positive creator identity.")
        if not isinstance(self.state, CoordinatorState):
            raise RuntimeError(f"SHM protocol v4 has an invalid coordinator state: {self.state}")


def _version() -> str:
    from flextensor_b200._version import __version__

    return __version__


def new_participant_id() -> int:
    return secrets.randbits(63) | 1


class Heartbeat:
    """One slot in ``{ns}_hb`` refreshed by a daemon thread."""

    def __init__(self, namespace: str, participant_id: int, lease_s: float = DEFAULT_LEASE_S):
        self.ns, self.pid_token, self.lease = namespace, participant_id, lease_s
        name = heartbeat_block_name(namespace)
        lock = ProcessFileLock(name)
        lock.acquire(timeout=30)
        try:
            try:
                self.seg = ShmSegment.create(name, _HB_SLOTS * _HB.size)
            except FileExistsError:
                self.seg = ShmSegment.attach(name)
            self.slot = self._claim()
        finally:
            lock.release()
        self._stop = threading.Event()
        self.beat()
        self._t = threading.Thread(target=self._run, name=f"ft-hb-{namespace}", daemon=True)
        self._t.start()

    def _claim(self) -> int:
        now = time.time()
        for i in range(_HB_SLOTS):
            pid, _, ts = _HB.unpack_from(self.seg.buf, i * _HB.size)
            if pid == 0 or now - ts > self.lease:
                _HB.pack_into(self.seg.buf, i * _HB.size, self.pid_token, os.getpid(), now)
                return i
        raise ShmCoordinatorError(f"no free heartbeat slot in {self.ns}")

    def beat(self) -> None:
        _HB.pack_into(self.seg.buf, self.slot * _HB.size, self.pid_token, os.getpid(), time.time())

    def _run(self) -> None:
        while not self._stop.wait(self.lease / 4):
            try:
                self.beat()
            except Exception:  # noqa: BLE001
                return

    def stop(self, clear: bool = True) -> None:
        self._stop.set()
        if clear:
            try:
                _HB.pack_into(self.seg.buf, self.slot * _HB.size, 0, 0, 0.0)
            except Exception:  # noqa: BLE001
                pass
        self.seg.close()


def last_beat(namespace: str, participant_id: int) -> float | None:
    name = heartbeat_block_name(namespace)
    if not shm_exists(name):
        return None
    seg = ShmSegment.attach(name)
    try:
        for i in range(_HB_SLOTS):
            pid, _, ts = _HB.unpack_from(seg.buf, i * _HB.size)
            if pid == participant_id:
                return ts
        return None
    finally:
        seg.close()


def live_participants(namespace: str, lease_s: float = DEFAULT_LEASE_S) -> int:
    name = heartbeat_block_name(namespace)
    if not shm_exists(name):
        return 0
    seg = ShmSegment.attach(name)
    try:
        now = time.time()
        n = 0
        for i in range(_HB_SLOTS):
            pid, _, ts = _HB.unpack_from(seg.buf, i * _HB.size)
            if pid and now - ts <= lease_s:
                n += 1
        return n
    finally:
        seg.close()


class ShmCoordinator:
    """Elect one creator per namespace; publish its plan; let followers wait for READY."""

    def __init__(self, namespace: str, lease_s: float = DEFAULT_LEASE_S, lock_timeout: float | None = 60.0):
        self.ns = namespace
        self.lease = lease_s
        self.participant_id = new_participant_id()
        self.heartbeat = Heartbeat(namespace, self.participant_id, lease_s)
        self.lock = ProcessFileLock(coord_block_name(namespace))
        self.lock.acquire(timeout=lock_timeout)
        try:
            name = coord_block_name(namespace)
            try:
                self.seg = ShmSegment.create(name, 4096)
                self.is_creator = True
                CoordBlockHeader(_version(), SHM_PROTOCOL_VERSION, self.participant_id,
                                 CoordinatorState.INITIALIZING).write_to(self.seg.buf)
            except FileExistsError:
                self.seg = ShmSegment.attach(name)
                self.is_creator = False
                hdr = self.header()
                stale = hdr.state != CoordinatorState.READY and not self._creator_alive(hdr)
                if stale:
                    # previous generation's creator died before READY: take over
                    logger.warning("namespace %s: abandoned generation found; taking over as creator", namespace)
                    self.is_creator = True
                    CoordBlockHeader(_version(), SHM_PROTOCOL_VERSION, self.participant_id,
                                     CoordinatorState.INITIALIZING).write_to(self.seg.buf)
        finally:
            self.lock.release()
        self._prof: ShmSegment | None = None

    # -------------------------------------------------------------- header
    def header(self) -> CoordBlockHeader:
        return CoordBlockHeader.read_from(self.seg.buf)

    def _creator_alive(self, hdr: CoordBlockHeader) -> bool:
        ts = last_beat(self.ns, hdr.creator_pid)
        return ts is not None and time.time() - ts <= self.lease

    # -------------------------------------------------------------- creator side
    def write_profile(self, payload: bytes) -> None:
        """Publish a length-prefixed state payload (``TensorManagerState.save_state_to_bytes``)."""
        if not self.is_creator:
            raise ShmCoordinatorError("only the creator publishes the profile")
        name = profile_block_name(self.ns)
        shm_unlink(name)
        self._prof = ShmSegment.create(name, len(payload))
        self._prof.buf[:len(payload)] = payload

    def notify_ready(self) -> None:
        h = self.header()
        h.state = CoordinatorState.READY
        h.write_to(self.seg.buf)

    def mark_failed(self, message: str) -> None:
        h = self.header()
        h.state = CoordinatorState.FAILED
        h.failure_message = message
        h.write_to(self.seg.buf)

    # -------------------------------------------------------------- follower side
    def wait_for_ready(self, timeout: float | None = None) -> None:
        deadline = None if not timeout else time.monotonic() + timeout
        while True:
            h = self.header()
            h.validate(_version(), SHM_PROTOCOL_VERSION)
            if h.state == CoordinatorState.READY:
                return
            if h.state == CoordinatorState.FAILED:
                raise ShmCreatorFailedError(f"creator failed: {h.failure_message}")
            if not self._creator_alive(h):
                raise ShmCreatorDiedError(f"creator of {self.ns} stopped heartbeating during INITIALIZING")
            if deadline is not None and time.monotonic() > deadline:
                raise TimeoutError(f"timed out after {timeout}s waiting for {self.ns} to become READY")
            time.sleep(POLL_S)

    def read_profile(self):
        from flextensor_b200.core.state import TensorManagerState

        seg = ShmSegment.attach(profile_block_name(self.ns))
        try:
            return TensorManagerState.load_state_from_bytes(bytes(seg.buf))
        finally:
            seg.close()

    # -------------------------------------------------------------- teardown
    def close(self, unlink_if_last: bool = True) -> None:
        self.heartbeat.stop()
        last = live_participants(self.ns, self.lease) == 0
        if self._prof is not None:
            self._prof.close()
        self.seg.close()
        if unlink_if_last and last:
            cleanup_namespace(self.ns)


def cleanup_namespace(namespace: str) -> list[str]:
    """Unlink every segment of a namespace (weights, profile, coord, store, heartbeat)."""
    from flextensor_b200.shm.segment import SHM_DIR

    removed = []
    try:
        names = os.listdir(SHM_DIR)
    except FileNotFoundError:
        return removed
    for n in names:
        if n.startswith(namespace + "_"):
            try:
                os.unlink(os.path.join(SHM_DIR, n))
                removed.append(n)
            except FileNotFoundError:
                pass
    return removed


def retire_abandoned(namespace: str, lease_s: float = DEFAULT_LEASE_S) -> bool:
    """Remove a namespace whose participants' leases all expired; True if removed."""
    if live_participants(namespace, lease_s) > 0:
        return False
    return bool(cleanup_namespace(namespace))
