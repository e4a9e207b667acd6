"""Every public kernel entry point of ``ops.api`` is re-exported by ``flextensor_b200.ops``, and
the model modules only call names that exist there (catches a missing export on CPU)."""

import ast
import inspect
import pathlib

import flextensor_b200.ops as ops
from flextensor_b200.ops import api

ROOT = pathlib.Path(__file__).resolve().parents[1] / "flextensor_b200"


def test_ops_reexports_api():
    public = {n for n, f in vars(api).items() if inspect.isfunction(f) and not n.startswith("_")
              and f.__module__ == api.__name__}
    missing = sorted(public - set(ops.__all__))
    assert not missing, f"not exported from flextensor_b200.ops: {missing}"


def test_models_use_existing_ops():
    used = set()
    for path in list((ROOT / "models").glob("*.py")) + list((ROOT / "parallel").glob("*.py")):
        for node in ast.walk(ast.parse(path.read_text())):
            if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id == "ops":
                used.add((path.name, node.attr))
    bad = [(f, a) for f, a in used if not hasattr(ops, a)]
    assert not bad, f"calls to missing ops: {bad}"


def test_flextensor_facade():
    import flextensor
    import flextensor_b200

    assert set(flextensor.__all__) == set(flextensor_b200.__all__)
    assert flextensor.offload is flextensor_b200.offload
    from flextensor.config import OffloadConfig

    assert OffloadConfig is flextensor_b200.OffloadConfig


def test_reference_vllm_class_paths():
    """The reference's vLLM class / module paths resolve to this package's classes."""
    pytest = __import__("pytest")
    pytest.importorskip("vllm")
    import importlib

    from flextensor_b200.contrib.vllm import loader, snapshot, worker

    assert importlib.import_module("flextensor.contrib.vllm.worker").FlexTensorOffloadWorker is \
        worker.FlexTensorOffloadWorker
    snap = importlib.import_module("flextensor.contrib.vllm.snapshot")
    assert snap.SnapshotWorker is snapshot.SnapshotWorker
    assert snap.FlexTensorSnapshotWorker is snapshot.FlexTensorSnapshotWorker
    assert importlib.import_module("flextensor.contrib.vllm.loader").FlexTensorModelLoader is \
        loader.FlexTensorModelLoader


def test_parallel_exports_resolve():
    """Every name in ``flextensor_b200.parallel.__all__`` resolves, and each parallelism strategy
    (context, tensor, expert, pipeline, striped streaming) has its entry point there."""
    import flextensor_b200.parallel as par

    missing = [n for n in par.__all__ if not hasattr(par, n)]
    assert not missing, missing
    for name in ("ContextParallel", "UlyssesAttention", "TPAllGather", "TPReduceScatter", "TPAllReduce",
                 "ExpertParallel", "PipelineStage", "split_stages", "pipeline_groups", "StripedTransferEngine"):
        assert name in par.__all__, name
