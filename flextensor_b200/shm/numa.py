"""NUMA placement of the shared host weight store.

On a multi-socket host every GPU streams its weights from one shared copy in ``/dev/shm``.
With the default first-touch policy all those pages land on the node of the process that
packed them, so the GPUs attached to the other sockets pull every byte across the socket
interconnect, and the node that holds the copy serves all copy engines at once. Spreading
the pages round-robin over the memory nodes (interleave) balances that load. The reference
gets the same effect by launching every worker under ``numactl --interleave=all``
(``examples/ltx23/outpaint/nginx_serve.sh:109-135``; measured there: 61.10 s -> 35.53 s per
49-frame request with eight single-GPU workers on eight NUMA nodes,
``examples/ltx23/outpaint/README.md:616-621``).

This module does it inside the library, with no ``numactl`` dependency:

* :func:`interleave_range` binds one mapping's pages (``mbind(MPOL_INTERLEAVE)``); the SHM
  weight store calls it on each segment it CREATES, before the first byte is written, so the
  policy is in place when the pages are first allocated (attaching processes never move
  pages that already exist);
* :func:`set_process_interleave` sets the calling process's default policy
  (``set_mempolicy``), the in-library form of ``numactl --interleave=all``;
* ``python -m flextensor_b200.shm.numa exec -- <cmd> ...`` runs a command under that policy
  (the serving launcher uses it when ``NUMA_INTERLEAVE=1``);
* :func:`range_policy` reads a mapping's policy back (``get_mempolicy(MPOL_F_ADDR)``).

The mode comes from ``FT_SHM_NUMA_INTERLEAVE``: ``0`` / unset = off (inherit whatever the
launcher set), ``1`` = on and strict (a refused ``mbind`` raises), ``auto`` = on where the
kernel allows it, else a warning.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import logging
import os
import platform
import sys

from flextensor_b200.config import _register_env_var

log = logging.getLogger(__name__)
_register_env_var("FT_SHM_NUMA_INTERLEAVE")

MPOL_DEFAULT = 0
MPOL_PREFERRED = 1
MPOL_BIND = 2
MPOL_INTERLEAVE = 3
MPOL_F_ADDR = 1 << 1

# syscall numbers (Linux): mbind, set_mempolicy, get_mempolicy
_SYSCALLS = {
    "x86_64": (237, 238, 239),
    "aarch64": (235, 237, 236),
}


class NumaUnavailable(OSError):
    pass


def _libc():
    return ctypes.CDLL(ctypes.util.find_library("c") or "libc.so.6", use_errno=True)


def _nr(which: int) -> int:
    arch = platform.machine()
    if arch not in _SYSCALLS:
        raise NumaUnavailable(f"NUMA syscalls are not wired for {arch}")
    return _SYSCALLS[arch][which]


def _parse_list(text: str) -> list[int]:
    """'0-3,8,10-11' -> [0, 1, 2, 3, 8, 10, 11]."""
    out: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            out.extend(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return out


def online_nodes() -> list[int]:
    try:
        with open("/sys/devices/system/node/online") as f:
            return _parse_list(f.read())
    except OSError:
        return [0]


def allowed_nodes() -> list[int]:
    """Memory nodes this process may allocate on (``Mems_allowed_list`` intersected with the
    online nodes)."""
    allowed = None
    try:
        with open("/proc/self/status") as f:
            for line in f:
                if line.startswith("Mems_allowed_list:"):
                    allowed = _parse_list(line.split(":", 1)[1])
                    break
    except OSError:
        pass
    online = online_nodes()
    if allowed is None:
        return online
    nodes = [n for n in allowed if n in online]
    return nodes or online


def _mask(nodes: list[int]):
    """(mask words, maxnode) for the kernel's nodemask argument."""
    if not nodes:
        raise ValueError("empty node list")
    bits = 64
    n_words = max(nodes) // bits + 1
    words = (ctypes.c_ulong * n_words)()
    for n in nodes:
        words[n // bits] |= 1 << (n % bits)
    return words, n_words * bits + 1


def interleave_range(addr: int, length: int, nodes: list[int] | None = None) -> None:
    """Interleave the pages of [addr, addr + length) over ``nodes`` (default: every allowed
    node). ``addr`` must be page aligned (an mmap base is). Pages already allocated keep
    their node; only pages touched later follow the policy."""
    nodes = nodes or allowed_nodes()
    words, maxnode = _mask(nodes)
    libc = _libc()
    r = libc.syscall(ctypes.c_long(_nr(0)), ctypes.c_void_p(addr), ctypes.c_ulong(length),
                     ctypes.c_int(MPOL_INTERLEAVE), words, ctypes.c_ulong(maxnode), ctypes.c_uint(0))
    if r != 0:
        e = ctypes.get_errno()
        raise NumaUnavailable(e, f"mbind(MPOL_INTERLEAVE, nodes={nodes}) refused: {os.strerror(e)}")


def set_process_interleave(nodes: list[int] | None = None) -> list[int]:
    """Make interleave the calling process's default policy for new pages; returns the nodes."""
    nodes = nodes or allowed_nodes()
    words, maxnode = _mask(nodes)
    libc = _libc()
    r = libc.syscall(ctypes.c_long(_nr(1)), ctypes.c_int(MPOL_INTERLEAVE), words, ctypes.c_ulong(maxnode))
    if r != 0:
        e = ctypes.get_errno()
        raise NumaUnavailable(e, f"set_mempolicy(MPOL_INTERLEAVE, nodes={nodes}) refused: {os.strerror(e)}")
    return nodes


def _get_policy(addr: int | None) -> tuple[int, list[int]]:
    words, maxnode = _mask([max(online_nodes())])
    for i in range(len(words)):
        words[i] = 0
    mode = ctypes.c_int(0)
    libc = _libc()
    r = libc.syscall(ctypes.c_long(_nr(2)), ctypes.byref(mode), words, ctypes.c_ulong(maxnode),
                     ctypes.c_void_p(addr or 0), ctypes.c_ulong(MPOL_F_ADDR if addr else 0))
    if r != 0:
        e = ctypes.get_errno()
        raise NumaUnavailable(e, f"get_mempolicy(MPOL_F_ADDR) refused: {os.strerror(e)}")
    nodes = [w * 64 + b for w in range(len(words)) for b in range(64) if words[w] >> b & 1]
    return mode.value, nodes


def range_policy(addr: int) -> tuple[int, list[int]]:
    """(policy, nodes) of the mapping that contains ``addr``."""
    return _get_policy(addr)


def process_policy() -> tuple[int, list[int]]:
    """(policy, nodes) of the calling thread's default policy."""
    return _get_policy(None)


def interleave_mode() -> str:
    """``off`` | ``on`` | ``auto`` from ``FT_SHM_NUMA_INTERLEAVE``."""
    v = os.environ.get("FT_SHM_NUMA_INTERLEAVE", "0").strip().lower()
    if v in ("", "0", "false", "off", "no"):
        return "off"
    if v == "auto":
        return "auto"
    if v in ("1", "true", "on", "yes"):
        return "on"
    raise ValueError(f"FT_SHM_NUMA_INTERLEAVE={v!r}: expected 0, 1 or auto")


def apply_to_new_mapping(addr: int, length: int, mode: str | None = None) -> bool:
    """Called by a segment's creator before the first write. Returns True if interleaved."""
    mode = mode or interleave_mode()
    if mode == "off" or length <= 0:
        return False
    try:
        interleave_range(addr, length)
        return True
    except NumaUnavailable as e:
        if mode == "on":
            raise
        log.warning("SHM NUMA interleave skipped: %s", e)
        return False


def _main(argv: list[str]) -> int:
    if len(argv) >= 2 and argv[0] == "exec" and argv[1] == "--" and len(argv) > 2:
        nodes = set_process_interleave()
        print(f"NUMA interleave over nodes {nodes}", file=sys.stderr)
        os.execvp(argv[2], argv[2:])
    if argv[:1] == ["probe"]:
        try:
            set_process_interleave()
            print("ok", allowed_nodes())
            return 0
        except NumaUnavailable as e:
            print(f"unavailable: {e}")
            return 1
    print("usage: python -m flextensor_b200.shm.numa exec -- <cmd> [args...] | probe", file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(_main(sys.argv[1:]))
