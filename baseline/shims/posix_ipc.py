"""Stand-in for ``posix_ipc`` (not in the offline wheelhouse): importable, unusable.

The benchmark configuration does not enable shared memory, so the reference
never calls into this module; any call raises immediately.
"""

O_CREAT = 0o100
O_EXCL = 0o200


class ExistentialError(Exception):
    pass


class BusyError(Exception):
    pass


def _unavailable(*_a, **_k):
    raise RuntimeError("posix_ipc is not installed on this machine (offline wheelhouse lacks it)")


Semaphore = SharedMemory = _unavailable
unlink_semaphore = unlink_shared_memory = _unavailable
