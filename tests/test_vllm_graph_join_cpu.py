"""The breakable-CUDA-graph segment join: vLLM's ``add_eager`` joins the offloader while a
capture runs (and only then), and installing twice wraps once."""

import importlib

import pytest

pytest.importorskip("vllm.compilation.breakable_cudagraph")


def test_add_eager_joins_the_offloader_only_while_capturing(monkeypatch):
    bc = importlib.import_module("vllm.compilation.breakable_cudagraph")
    base = importlib.import_module("vllm.model_executor.offloader.base")
    from flextensor_b200.contrib.vllm import graph_join

    calls = []

    class FakeOffloader:
        def join_after_forward(self):
            calls.append("join")

    def fake_add_eager(self, fn):
        calls.append("eager")
        return fn()

    monkeypatch.setattr(bc.BreakableCUDAGraphCapture, "add_eager", fake_add_eager)
    monkeypatch.setattr(base, "get_offloader", lambda: FakeOffloader())
    assert graph_join.install_segment_join()
    assert graph_join.install_segment_join()  # idempotent: one wrapper
    cap = object.__new__(bc.BreakableCUDAGraphCapture)
    cap._capturing = True
    assert bc.BreakableCUDAGraphCapture.add_eager(cap, lambda: 7) == 7
    assert calls == ["join", "eager"]
    calls.clear()
    cap._capturing = False
    bc.BreakableCUDAGraphCapture.add_eager(cap, lambda: None)
    assert calls == ["eager"]
