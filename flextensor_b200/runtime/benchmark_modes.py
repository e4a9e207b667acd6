"""TorchFunctionMode debugging/benchmark modes (``src/flextensor/benchmark_tensor_mode.py:18-312``).

* :class:`TensorBenchmarkMode` -- base: counts every intercepted torch call and
  the host-side time spent inside it, keyed by function name.
* :class:`BenchmarkReplace` -- replaces CPU tensor arguments with device copies
  on the fly (trace/debug path for models that read weights outside any trap)
  and counts the bytes it moved.
* :class:`PreloadToDevice` -- moves a model to the device once on entry (the
  ``enabled=False`` path) and passes calls through.
* :class:`NoOpBenchmark` -- passes everything through.

:class:`TraceTensor` (``src/flextensor/tensor.py:9-51``) marks a tensor as managed by the
runtime (the ``_use_trace_tensor`` debug path): results of out-of-place ops on it are plain
tensors, so the mark never spreads to activations, while in-place ops keep it.
``BenchmarkReplace(trace=True)`` returns its device copies as TraceTensors and records, per
source tensor, its size and the median time of its host -> device copy.
"""

from __future__ import annotations

import time
from collections import defaultdict

import torch
from torch.overrides import TorchFunctionMode


class TensorBenchmarkMode(TorchFunctionMode):
    def __init__(self, device: torch.device | str | None = None):
        super().__init__()
        self.device = torch.device(device) if device is not None else None
        self.calls: dict[str, int] = defaultdict(int)
        self.host_ms: dict[str, float] = defaultdict(float)

    def transform(self, x):
        return x

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        name = getattr(func, "__name__", str(func))
        args = torch.utils._pytree.tree_map(self.transform, args)
        kwargs = torch.utils._pytree.tree_map(self.transform, kwargs)
        t0 = time.perf_counter()
        out = func(*args, **kwargs)
        self.calls[name] += 1
        self.host_ms[name] += (time.perf_counter() - t0) * 1e3
        return out


class TraceTensor(torch.Tensor):
    @staticmethod
    def __new__(cls, data: torch.Tensor, name: str | None = None):
        t = torch.Tensor._make_subclass(cls, data, data.requires_grad)
        t.trace_name = name
        return t

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        res = super().__torch_function__(func, types, args, kwargs or {})
        if getattr(func, "__name__", "").endswith("_"):
            return res  # in-place: the traced tensor itself
        if isinstance(res, TraceTensor):
            return res.as_subclass(torch.Tensor)
        return res


def wrap_trace_tensor(t, name: str | None = None):
    if isinstance(t, TraceTensor) or not isinstance(t, torch.Tensor):
        return t
    return TraceTensor(t, name)


def is_trace_tensor(t) -> bool:
    return isinstance(t, TraceTensor)


class BenchmarkReplace(TensorBenchmarkMode):
    def __init__(self, device: torch.device | str, trace: bool = False, reps: int = 3):
        super().__init__(device)
        self.moved_bytes = 0
        self.trace = trace
        self.reps = reps
        self._cache: dict[int, torch.Tensor] = {}
        self.tensor_stats: dict[int, dict] = {}  # host data_ptr -> {bytes, load_ms}

    def _timed_copy(self, x: torch.Tensor) -> tuple[torch.Tensor, float]:
        times = []
        d = None
        for _ in range(max(1, self.reps)):
            if self.device.type == "cuda":
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                d = x.to(self.device, non_blocking=True)
                b.record()
                b.synchronize()
                times.append(a.elapsed_time(b))
            else:
                t0 = time.perf_counter()
                d = x.to(self.device)
                times.append((time.perf_counter() - t0) * 1e3)
        times.sort()
        return d, times[len(times) // 2]

    def transform(self, x):
        if isinstance(x, torch.Tensor) and x.device.type == "cpu" and self.device is not None \
                and self.device.type != "cpu" and not x.is_meta:
            key = x.data_ptr()
            d = self._cache.get(key)
            if d is None:
                if self.trace:
                    d, ms = self._timed_copy(x)
                    d = wrap_trace_tensor(d)
                    self.tensor_stats[key] = {"bytes": x.numel() * x.element_size(), "load_ms": ms}
                else:
                    d = x.to(self.device, non_blocking=True)
                self._cache[key] = d
                self.moved_bytes += x.numel() * x.element_size()
            return d
        return x


class PreloadToDevice(TensorBenchmarkMode):
    def __init__(self, model: torch.nn.Module, device: torch.device | str):
        super().__init__(device)
        self.model = model

    def __enter__(self):
        self.model.to(self.device)
        return super().__enter__()


class NoOpBenchmark(TensorBenchmarkMode):
    pass
