"""Cross-process synchronisation primitives on ``/dev/shm`` files (no posix_ipc dependency).

Parity with ``src/flextensor/shm/sync_primitives.py`` (``SemaphoreLock``) and
``shm/multiprocess_condition.py`` (``SharedMultiString``, ``MultiprocessCondition``):

* :class:`SemaphoreLock` -- a counting semaphore of ``slots`` permits. Each permit is an
  ``fcntl`` byte-range lock on one byte of a lock file, so a permit held by a process that
  dies is released by the kernel (a POSIX named semaphore would stay decremented forever).
* :class:`SharedMultiString` -- an append-only journal of names (e.g. the segments a session
  owns) with a ready marker; writers serialise on a file lock; readers see complete records.
* :class:`MultiprocessCondition` -- one-shot "ready" condition: ``notify_ready`` publishes,
  ``wait_for_ready`` polls with backoff until it is set or the timeout passes.

Every wait is bounded (``timeout``); nothing here spins without a limit.
"""

from __future__ import annotations

import errno
import fcntl
import os
import struct
import time

from flextensor_b200.shm.segment import ProcessFileLock, shm_path


class SemaphoreLock:
    def __init__(self, name: str, slots: int = 1):
        if slots < 1:
            raise ValueError("slots must be >= 1")
        self.name, self.slots = name, slots
        self.path = shm_path(name) + ".sem"
        self._fd = os.open(self.path, os.O_RDWR | os.O_CREAT, 0o600)
        if os.fstat(self._fd).st_size < slots:
            os.ftruncate(self._fd, slots)
        self._held: int | None = None

    def _try(self, i: int) -> bool:
        try:
            fcntl.lockf(self._fd, fcntl.LOCK_EX | fcntl.LOCK_NB, 1, i, os.SEEK_SET)
            return True
        except OSError as e:
            if e.errno in (errno.EAGAIN, errno.EACCES):
                return False
            raise

    def acquire(self, non_blocking: bool = False, timeout: float | None = None) -> None:
        if self._held is not None:
            raise RuntimeError("this handle already holds a permit")
        deadline = None if timeout is None else time.monotonic() + timeout
        delay = 0.001
        while True:
            for i in range(self.slots):
                if self._try(i):
                    self._held = i
                    return
            if non_blocking:
                raise BlockingIOError(f"no free permit on {self.path}")
            if deadline is not None and time.monotonic() >= deadline:
                raise TimeoutError(f"timed out waiting for a permit on {self.path}")
            time.sleep(delay)
            delay = min(delay * 2, 0.05)

    def release(self) -> None:
        if self._held is None:
            raise RuntimeError("release() without a held permit")
        fcntl.lockf(self._fd, fcntl.LOCK_UN, 1, self._held, os.SEEK_SET)
        self._held = None

    signal = release

    def __enter__(self):
        self.acquire()
        return self

    def __exit__(self, *exc):
        self.release()

    def close(self) -> None:
        if self._fd >= 0:
            if self._held is not None:
                self.release()
            os.close(self._fd)
            self._fd = -1

    def unlink(self) -> None:
        self.close()
        self.unlink_name()

    def unlink_name(self) -> None:
        try:
            os.unlink(self.path)
        except FileNotFoundError:
            pass


class SharedMultiString:
    """Records: u32 length + utf-8 bytes, appended under a file lock; a ``.ready`` marker file."""

    def __init__(self, name: str):
        self.name = name
        self.path = shm_path(name) + ".journal"
        self.ready_path = shm_path(name) + ".ready"
        self._lock = ProcessFileLock(name + ".journal")
        with open(self.path, "ab"):
            pass

    def append(self, string: str) -> None:
        data = string.encode("utf-8")
        with self._lock:
            with open(self.path, "ab") as f:
                f.write(struct.pack("<I", len(data)) + data)
                f.flush()
                os.fsync(f.fileno())

    def set_ready(self) -> None:
        with open(self.ready_path, "wb") as f:
            f.write(b"1")

    def is_ready(self) -> bool:
        return os.path.exists(self.ready_path)

    def get_list(self) -> list[str]:
        out: list[str] = []
        with open(self.path, "rb") as f:
            blob = f.read()
        i = 0
        while i + 4 <= len(blob):
            (n,) = struct.unpack_from("<I", blob, i)
            if i + 4 + n > len(blob):
                break  # a record still being written
            out.append(blob[i + 4:i + 4 + n].decode("utf-8"))
            i += 4 + n
        return out

    def close(self) -> None:
        self._lock.release()

    def unlink_name(self) -> None:
        for p in (self.path, self.ready_path):
            try:
                os.unlink(p)
            except FileNotFoundError:
                pass
        self._lock.unlink()

    def unlink(self) -> None:
        self.close()
        self.unlink_name()


class MultiprocessCondition:
    def __init__(self, name: str):
        self.name = name
        self._ready = SharedMultiString(name + ".cond")

    def notify_ready(self, note: str = "") -> None:
        if note:
            self._ready.append(note)
        self._ready.set_ready()

    def wait_for_ready(self, timeout: float = 60.0) -> list[str]:
        deadline = time.monotonic() + timeout
        delay = 0.001
        while not self._ready.is_ready():
            if time.monotonic() >= deadline:
                raise TimeoutError(f"condition {self.name!r} not signalled within {timeout:.1f}s")
            time.sleep(delay)
            delay = min(delay * 2, 0.05)
        return self._ready.get_list()

    def close(self) -> None:
        self._ready.close()

    def unlink(self) -> None:
        self._ready.unlink()

    unlink_names = unlink
