"""TorchFunctionMode debugging/benchmark modes (``src/flextensor/benchmark_tensor_mode.py:18-312``).

* :class:`TensorBenchmarkMode` -- base: counts every intercepted torch call and
  the host-side time spent inside it, keyed by function name.
* :class:`BenchmarkReplace` -- replaces CPU tensor arguments with device copies
  on the fly (trace/debug path for models that read weights outside any trap)
  and counts the bytes it moved.
* :class:`PreloadToDevice` -- moves a model to the device once on entry (the
  ``enabled=False`` path) and passes calls through.
* :class:`NoOpBenchmark` -- passes everything through.
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


class BenchmarkReplace(TensorBenchmarkMode):
    def __init__(self, device: torch.device | str):
        super().__init__(device)
        self.moved_bytes = 0
        self._cache: dict[int, torch.Tensor] = {}

    def transform(self, x):
        if isinstance(x, torch.Tensor) and x.device.type == "cpu" and self.device is not None \
                and self.device.type != "cpu":
            key = x.data_ptr()
            d = self._cache.get(key)
            if d is None:
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
