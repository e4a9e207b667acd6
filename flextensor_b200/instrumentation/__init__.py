"""Constructor-argument instrumentation (parity with ``flextensor/instrumentation/__init__.py``).

Classes decorated with :func:`instrumentable` record their ``__init__`` arguments into a
process-wide registry while it is enabled. ``dump_to_file`` / ``dump_to_directory`` write
the records plus a host-memory snapshot as one JSON document with the keys
``timestamp``, ``flextensor_version``, ``components`` and ``host_memory`` (the same keys as
the reference, so its analysis scripts read our dumps). The OffloadManager dumps once on
entering INFERENCE when ``OffloadConfig.enable_instrumentation`` is set, adding
``memory_transfer_stats`` (the H2D size->ms table).
"""

from __future__ import annotations

from typing import Any

from flextensor_b200.instrumentation.core import (
    ComponentRecord,
    InstrumentationRegistry,
    capture_host_resources,
    dump_to_directory,
    dump_to_file,
    instrumentable,
    serialize_args,
    serialize_value,
)

__all__ = [
    "ComponentRecord",
    "InstrumentationRegistry",
    "capture_host_resources",
    "dump_instrumentation",
    "dump_to_directory",
    "dump_to_file",
    "get_registry",
    "instrumentable",
    "serialize_args",
    "serialize_value",
]


def get_registry() -> InstrumentationRegistry:
    return InstrumentationRegistry.get_instance()


def dump_instrumentation(output_dir: str, *, extra: dict[str, Any] | None = None):
    return dump_to_directory(output_dir, extra=extra)
