"""Shared resident-tensor store, format FTTS v1 (interop format of
``src/flextensor/shm/tensor_store.py:33-288``).

Layout of segment ``{ns}_t``:

* header ``<4sIQQQ`` = (b"FTTS", 1, manifest length, data offset, data size);
* manifest: sorted-key compact JSON ``{"tensors": [{aliases, dtype, kind,
  payload_offset, persistent, requires_grad, shape, stride}, ...]}``;
* data at a 64-byte aligned offset; each payload at max(8, itemsize) alignment.

The creator publishes the resident parameters it names plus every buffer;
followers (which build the model on ``meta``) validate the header and copy
each entry to their device, rebinding all aliases of the same object.
"""

from __future__ import annotations

import json
import struct

import torch
from torch import nn

from flextensor_b200.shm.namespace import tensor_store_name
from flextensor_b200.shm.segment import ShmSegment, shm_unlink

MAGIC = b"FTTS"
VERSION = 1
_HDR = struct.Struct("<4sIQQQ")
DATA_ALIGN = 64
PAYLOAD_ALIGN = 8


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def _dtype_name(d: torch.dtype) -> str:
    return str(d).replace("torch.", "")


def _dtype_from(name: str) -> torch.dtype:
    d = getattr(torch, name, None)
    if not isinstance(d, torch.dtype):
        raise ValueError(f"unknown dtype {name!r}")
    return d


def _persistent(model: nn.Module, alias: str) -> bool:
    mod_path, _, leaf = alias.rpartition(".")
    mod = model.get_submodule(mod_path) if mod_path else model
    return leaf not in mod._non_persistent_buffers_set


def plan_manifest(model: nn.Module, parameter_names: list[str]):
    params = dict(model.named_parameters(remove_duplicate=False))
    bufs = dict(model.named_buffers(remove_duplicate=False))
    entries, sources = [], []
    chosen: dict[int, list[str]] = {}
    for n in parameter_names:
        if n not in params:
            raise ValueError(f"SharedTensorStore requested parameter {n!r} is not a registered parameter")
        chosen.setdefault(id(params[n]), [])
    for n, p in params.items():
        if id(p) in chosen:
            chosen[id(p)].append(n)
    objs = [("parameter", tuple(a), params[a[0]]) for a in chosen.values()]
    seen: dict[int, list[str]] = {}
    for n, b in bufs.items():
        seen.setdefault(id(b), []).append(n)
    objs += [("buffer", tuple(a), bufs[a[0]]) for a in seen.values()]
    cur = 0
    for kind, aliases, t in objs:
        t = t.detach()
        off = _align(cur, max(PAYLOAD_ALIGN, t.element_size()))
        nbytes = t.numel() * t.element_size()
        stride = [1] * t.dim()
        for i in range(t.dim() - 2, -1, -1):
            stride[i] = stride[i + 1] * t.shape[i + 1]
        entries.append({
            "aliases": list(aliases), "dtype": _dtype_name(t.dtype), "kind": kind, "payload_offset": off,
            "persistent": None if kind == "parameter" else [_persistent(model, a) for a in aliases],
            "requires_grad": bool(t.requires_grad) if kind == "parameter" else False,
            "shape": list(t.shape), "stride": stride,
        })
        sources.append(t)
        cur = off + nbytes
    manifest = json.dumps({"tensors": entries}, sort_keys=True, separators=(",", ":")).encode()
    data_off = _align(_HDR.size + len(manifest), DATA_ALIGN)
    return entries, sources, manifest, data_off, cur


class SharedTensorStore:
    def __init__(self, seg: ShmSegment, entries: list[dict], data_offset: int):
        self.seg, self.entries, self.data_offset = seg, entries, data_offset

    @classmethod
    def create_from_model(cls, namespace: str, model: nn.Module, parameter_names: list[str]) -> "SharedTensorStore":
        entries, sources, manifest, data_off, data_size = plan_manifest(model, parameter_names)
        name = tensor_store_name(namespace)
        shm_unlink(name)
        seg = ShmSegment.create(name, data_off + data_size)
        _HDR.pack_into(seg.buf, 0, MAGIC, VERSION, len(manifest), data_off, data_size)
        seg.buf[_HDR.size:_HDR.size + len(manifest)] = manifest
        raw = seg.tensor()
        for e, t in zip(entries, sources):
            n = t.numel() * t.element_size()
            if n:
                dst = raw[data_off + e["payload_offset"]:data_off + e["payload_offset"] + n]
                dst.view(t.dtype).view(t.shape).copy_(t.to("cpu"))
        return cls(seg, entries, data_off)

    @classmethod
    def attach(cls, namespace: str) -> "SharedTensorStore":
        seg = ShmSegment.attach(tensor_store_name(namespace))
        magic, ver, mlen, data_off, data_size = _HDR.unpack_from(seg.buf, 0)
        if magic != MAGIC or ver != VERSION:
            seg.close()
            raise ValueError(f"not an FTTS v{VERSION} store (magic={magic!r}, version={ver})")
        if data_off < _HDR.size + mlen or data_off + data_size > seg.size:
            seg.close()
            raise ValueError("corrupt FTTS store bounds")
        manifest = json.loads(bytes(seg.buf[_HDR.size:_HDR.size + mlen]))
        return cls(seg, manifest["tensors"], data_off)

    def tensor(self, e: dict) -> torch.Tensor:
        d = _dtype_from(e["dtype"])
        shape = tuple(e["shape"])
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.empty((), dtype=d).element_size()
        raw = self.seg.tensor()[self.data_offset + e["payload_offset"]:self.data_offset + e["payload_offset"] + nbytes]
        return raw.view(d).view(shape)

    def materialize_into(self, model: nn.Module, device: torch.device | str) -> None:
        for e in self.entries:
            src = self.tensor(e).to(device)
            if device == "cpu" or str(device) == "cpu":
                src = src.clone()  # never alias the shared mapping from a live module
            obj = nn.Parameter(src, requires_grad=e["requires_grad"]) if e["kind"] == "parameter" else None
            for alias in e["aliases"]:
                mod_path, _, leaf = alias.rpartition(".")
                mod = model.get_submodule(mod_path) if mod_path else model
                if obj is not None:
                    setattr(mod, leaf, obj)
                else:
                    mod.register_buffer(leaf, src, persistent=bool(e["persistent"][0]) if e["persistent"] else True)

    def close(self) -> None:
        self.seg.close()
