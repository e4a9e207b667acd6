"""Cross-process synchronisation primitives on ``/dev/shm`` files (no posix_ipc dependency).

Parity with ``src/flextensor/shm/sync_primitives.py`` (``SemaphoreLock``) and
``shm/multiprocess_condition.py`` (``SharedMultiString``, ``MultiprocessCondition``):

* :class:`SemaphoreLock` -- a counting semaphore of ``slots`` permits. Each permit is a
  ``flock`` on its own file taken through a descriptor opened for that acquire, so handles
  and threads in one process contend like processes do, and a permit held by a process that
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
import threading
import time

from flextensor_b200.shm.segment import ProcessFileLock, shm_path


class SemaphoreLock:
    """Counting semaphore of ``slots`` permits shared by every process that opens ``name``.

    Permit ``i`` is an exclusive ``flock`` on its own file ``<name>.sem.<i>``, taken on a file
    descriptor opened for that one acquire. ``flock`` locks belong to the open file
    description, not to the process, so two handles in one process, or two threads sharing a
    handle, contend for permits exactly as two processes do, and closing one descriptor frees
    only the permit taken through it. A permit held by a process that dies is released by the
    kernel. One handle may hold several permits (one per acquire, e.g. from several threads);
    ``release`` returns the most recent one.
    """

    def __init__(self, name: str, slots: int = 1):
        if slots < 1:
            raise ValueError("slots must be >= 1")
        self.name, self.slots = name, slots
        self.path = shm_path(name) + ".sem"
        fd = os.open(self.path, os.O_RDWR | os.O_CREAT, 0o600)  # marker: lets unlink find the set
        os.close(fd)
        self._permits = [f"{self.path}.{i}" for i in range(slots)]
        self._held: list[tuple[int, int]] = []  # (permit index, fd holding its flock)
        self._mutex = threading.Lock()
        self._closed = False

    def _try(self, i: int) -> int:
        fd = os.open(self._permits[i], os.O_RDWR | os.O_CREAT, 0o600)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX | fcntl.LOCK_NB)
            return fd
        except OSError as e:
            os.close(fd)
            if e.errno in (errno.EAGAIN, errno.EACCES, errno.EWOULDBLOCK):
                return -1
            raise

    def acquire(self, non_blocking: bool = False, timeout: float | None = None) -> None:
        if self._closed:
            raise RuntimeError(f"semaphore {self.name!r} is closed")
        deadline = None if timeout is None else time.monotonic() + timeout
        delay = 0.001
        while True:
            for i in range(self.slots):
                fd = self._try(i)
                if fd >= 0:
                    with self._mutex:
                        self._held.append((i, fd))
                    return
            if non_blocking:
                raise BlockingIOError(f"no free permit on {self.path}")
            if deadline is not None and time.monotonic() >= deadline:
                raise TimeoutError(f"timed out waiting for a permit on {self.path}")
            time.sleep(delay)
            delay = min(delay * 2, 0.05)

    def release(self) -> None:
        with self._mutex:
            if not self._held:
                raise RuntimeError("release() without a held permit")
            _, fd = self._held.pop()
        fcntl.flock(fd, fcntl.LOCK_UN)
        os.close(fd)

    signal = release

    @property
    def held(self) -> int:
        """Permits this handle holds now."""
        with self._mutex:
            return len(self._held)

    def __enter__(self):
        self.acquire()
        return self

    def __exit__(self, *exc):
        self.release()

    def close(self) -> None:
        """Release the permits this handle holds (no other handle's) and retire the handle."""
        while self.held:
            self.release()
        self._closed = True

    def unlink(self) -> None:
        self.close()
        self.unlink_name()

    def unlink_name(self) -> None:
        for p in [*self._permits, self.path]:
            try:
                os.unlink(p)
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
