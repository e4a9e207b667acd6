"""POSIX shared-memory segments and inter-process locks, without third-party packages.

A segment is a file under ``/dev/shm`` (what ``shm_open`` creates on Linux)
opened with ``O_CREAT|O_EXCL`` by its creator and mapped with ``mmap``; any
process that knows the name attaches to the same pages. Locks are ``fcntl``
advisory locks on a lock file (released by the kernel if the holder dies, so a
crashed creator can never wedge an election).

NUMA: with ``FT_SHM_NUMA_INTERLEAVE=1`` (or ``auto``) a creator interleaves its segment's
pages over the memory nodes before writing them (``flextensor_b200.shm.numa``).

Pinning: ``pin()`` page-locks the mapping in place with ``cudaHostRegister``
(native helper) so every local worker's copy engine DMAs from the SAME host
pages -- one host copy of the weights for all ranks.
"""

from __future__ import annotations

import errno
import fcntl
import mmap
import os
import time

import torch

SHM_DIR = os.environ.get("FLEXTENSOR_B200_SHM_DIR", "/dev/shm")


def shm_path(name: str) -> str:
    return os.path.join(SHM_DIR, name.lstrip("/"))


def shm_exists(name: str) -> bool:
    return os.path.exists(shm_path(name))


def shm_unlink(name: str) -> bool:
    try:
        os.unlink(shm_path(name))
        return True
    except FileNotFoundError:
        return False


class ShmSegment:
    def __init__(self, name: str, size: int, create: bool):
        self.name = name.lstrip("/")
        self.path = shm_path(self.name)
        self.created = create
        self._tensor = None
        flags = os.O_RDWR | (os.O_CREAT | os.O_EXCL if create else 0)
        self._fd = os.open(self.path, flags, 0o600)
        try:
            if create:
                os.ftruncate(self._fd, max(size, 1))
            self.size = os.fstat(self._fd).st_size if not create else max(size, 1)
            self._mm = mmap.mmap(self._fd, self.size, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
            self.numa_interleaved = False
            if create:
                # before the first write: the pages take the policy when they are first allocated
                from flextensor_b200.shm.numa import apply_to_new_mapping

                self.numa_interleaved = apply_to_new_mapping(self.tensor().data_ptr(), self.size)
        except BaseException:
            os.close(self._fd)
            if create:
                shm_unlink(self.name)
            raise
        self._pinned_ptr = 0

    @classmethod
    def create(cls, name: str, size: int) -> "ShmSegment":
        return cls(name, size, True)

    @classmethod
    def attach(cls, name: str) -> "ShmSegment":
        return cls(name, 0, False)

    @property
    def buf(self) -> memoryview:
        if self._mm is None:
            raise ValueError(f"segment {self.name} is closed")
        return memoryview(self._mm)

    def tensor(self) -> torch.Tensor:
        if self._tensor is None:
            self._tensor = torch.frombuffer(self._mm, dtype=torch.uint8, count=self.size)
        return self._tensor

    def pin(self) -> None:
        if self._pinned_ptr or not torch.cuda.is_available():
            return
        from flextensor_b200.ops import native

        t = self.tensor()
        native.host_register(t.data_ptr(), t.numel())
        self._pinned_ptr = t.data_ptr()

    def close(self) -> None:
        if self._pinned_ptr:
            from flextensor_b200.ops import native

            try:
                native.host_unregister(self._pinned_ptr)
            finally:
                self._pinned_ptr = 0
        # Drop our references only: tensors created by tensor() keep the mmap object
        # alive, and the pages are unmapped when the last of them is freed. Closing
        # the mapping here would leave such tensors pointing at unmapped memory.
        self._tensor = None
        self._mm = None
        if self._fd >= 0:
            os.close(self._fd)
            self._fd = -1

    def unlink(self) -> None:
        shm_unlink(self.name)


class ProcessFileLock:
    """fcntl lock on ``<SHM_DIR>/<name>.lock``; bounded acquisition with a timeout."""

    def __init__(self, name: str):
        self.path = shm_path(name) + ".lock"
        self._fd = -1

    def acquire(self, timeout: float | None = None, poll: float = 0.01) -> None:
        fd = os.open(self.path, os.O_RDWR | os.O_CREAT, 0o600)
        deadline = None if not timeout else time.monotonic() + timeout
        while True:
            try:
                fcntl.flock(fd, fcntl.LOCK_EX | fcntl.LOCK_NB)
                self._fd = fd
                return
            except OSError as e:
                if e.errno not in (errno.EAGAIN, errno.EACCES):
                    os.close(fd)
                    raise
            if deadline is not None and time.monotonic() > deadline:
                os.close(fd)
                raise TimeoutError(f"timed out acquiring {self.path}")
            time.sleep(poll)

    def release(self) -> None:
        if self._fd >= 0:
            fcntl.flock(self._fd, fcntl.LOCK_UN)
            os.close(self._fd)
            self._fd = -1

    def __enter__(self):
        self.acquire()
        return self

    def __exit__(self, *exc):
        self.release()

    def unlink(self) -> None:
        try:
            os.unlink(self.path)
        except FileNotFoundError:
            pass
