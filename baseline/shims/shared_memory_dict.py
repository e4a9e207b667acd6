"""Stand-in for ``shared-memory-dict`` (not in the offline wheelhouse): importable, unusable."""


class SharedMemoryDict(dict):
    def __init__(self, *_a, **_k):
        raise RuntimeError("shared_memory_dict is not installed on this machine (offline wheelhouse lacks it)")
