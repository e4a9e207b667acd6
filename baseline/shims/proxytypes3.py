"""Stand-in for the third-party ``proxytypes3`` package (not in the offline wheelhouse).

Only ``ObjectWrapper`` is provided: a transparent proxy whose wrapped object
lives in ``__subject__`` and receives every attribute read/write. The
reference's ``OffloadModelProxy`` subclasses it and overrides ``__call__``/
``forward`` itself, so this is all its stock code path uses.
"""


class ObjectWrapper:
    __slots__ = ("__subject__", "__dict__")

    def __init__(self, obj):
        object.__setattr__(self, "__subject__", obj)

    def __getattr__(self, name):
        return getattr(object.__getattribute__(self, "__subject__"), name)

    def __setattr__(self, name, value):
        if name == "__subject__":
            object.__setattr__(self, name, value)
        else:
            setattr(object.__getattribute__(self, "__subject__"), name, value)

    def __delattr__(self, name):
        delattr(object.__getattribute__(self, "__subject__"), name)

    def __repr__(self):
        return repr(object.__getattribute__(self, "__subject__"))
