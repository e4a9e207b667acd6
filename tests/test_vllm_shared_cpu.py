"""vLLM data-parallel replicas sharing one host weight copy (``contrib/vllm/shared.py``): the
fail-closed topology check, the creator / follower load flow against a fake shared session, the
follower's storage-identity check, and the ``flextensor_shm`` loader registration. CPU only."""

from types import SimpleNamespace

import pytest
import torch
from torch import nn

from flextensor_b200.contrib.vllm import shared as S


def _cfgs(**over):
    mc = SimpleNamespace(runner_type="generate", convert_type="none", quantization=None)
    par = SimpleNamespace(tensor_parallel_size=1, pipeline_parallel_size=1, prefill_context_parallel_size=1,
                          decode_context_parallel_size=1, data_parallel_backend="mp", nnodes=1,
                          data_parallel_external_lb=False, data_parallel_hybrid_lb=False,
                          enable_expert_parallel=False, enable_eplb=False, enable_ep_weight_filter=False)
    vc = SimpleNamespace(model_config=mc, parallel_config=par, lora_config=None, speculative_config=None,
                         load_config=SimpleNamespace(load_format="auto"))
    cfg = SimpleNamespace(profile_storage_dir="/tmp/p", profile_read_only=True, shm_namespace="ns")
    for k, v in over.items():
        obj, attr = k.split(".")
        setattr({"mc": mc, "par": par, "vc": vc, "cfg": cfg, "lc": vc.load_config}[obj], attr, v)
    return vc, cfg


def test_valid_topology_passes():
    S.validate_shared_topology(*_cfgs())


@pytest.mark.parametrize("override", [
    {"cfg.profile_read_only": False}, {"cfg.profile_storage_dir": None}, {"cfg.shm_namespace": None},
    {"mc.quantization": "fp8"}, {"mc.runner_type": "pooling"}, {"vc.lora_config": object()},
    {"vc.speculative_config": object()}, {"par.tensor_parallel_size": 2}, {"par.pipeline_parallel_size": 2},
    {"par.decode_context_parallel_size": 2}, {"par.data_parallel_backend": "ray"}, {"par.nnodes": 2},
    {"par.data_parallel_external_lb": True}, {"par.enable_expert_parallel": True}, {"lc.load_format": "dummy"}])
def test_unsupported_topologies_fail_closed(override):
    with pytest.raises(S.SharedTopologyError):
        S.validate_shared_topology(*_cfgs(**override))


class _FakeSession:
    """Plays the shared session: the creator runs the checkpoint factory, a follower the meta
    factory and then 'materialises' the model from the store (here: fresh CPU tensors)."""

    def __init__(self, creator: bool):
        self.creator = creator
        self.calls = []

    def offload_from_profile(self, profile_directory, *, config, name, creator_model_factory,
                             follower_model_factory, materialize_device):
        self.calls.append((profile_directory, name, str(materialize_device)))
        if self.creator:
            return creator_model_factory()
        m = follower_model_factory()
        return m.to_empty(device="cpu")


def _ctx(session):
    return S.SharedLoad(session=session, config=object(), profile_directory="/p", device=torch.device("cpu"),
                        underlying_format="auto", manager_name="vllm")


def test_creator_loads_the_checkpoint():
    ctx = _ctx(_FakeSession(creator=True))
    model = S.shared_load(ctx, lambda: nn.Linear(4, 4), lambda: pytest.fail("meta build on the creator"),
                          lambda m: pytest.fail("follower hook on the creator"))
    assert ctx.role == "creator" and ctx.model is model
    assert ctx.session.calls == [("/p", "vllm", "cpu")]


def test_follower_builds_meta_and_keeps_shared_storage():
    ctx = _ctx(_FakeSession(creator=False))

    def meta():
        with torch.device("meta"):
            return nn.Sequential(nn.Linear(4, 4), nn.LayerNorm(4))

    seen = []
    model = S.shared_load(ctx, lambda: pytest.fail("checkpoint on a follower"), meta, lambda m: seen.append(m))
    assert ctx.role == "follower" and seen == [model]


def test_follower_hook_that_moves_storage_is_rejected():
    ctx = _ctx(_FakeSession(creator=False))

    def meta():
        with torch.device("meta"):
            return nn.Linear(4, 4)

    def bad_hook(m):
        m.weight.data = m.weight.data.clone()  # new storage behind the same parameter

    with pytest.raises(RuntimeError, match="shared storage"):
        S.shared_load(ctx, lambda: None, meta, bad_hook)


def test_follower_skeleton_must_be_meta():
    ctx = _ctx(_FakeSession(creator=False))
    with pytest.raises(RuntimeError, match="concrete tensors"):
        S.shared_load(ctx, lambda: None, lambda: nn.Linear(2, 2), lambda m: None)


def test_one_active_load_per_context():
    ctx = _ctx(_FakeSession(creator=True))
    with S.active_shared_load(ctx):
        with pytest.raises(RuntimeError):
            with S.active_shared_load(ctx):
                pass


def test_shared_loader_registered_with_vllm():
    pytest.importorskip("vllm")
    from vllm.model_executor import model_loader

    assert S.FlexTensorSharedLoader is not None
    assert model_loader._LOAD_FORMAT_TO_MODEL_LOADER[S.SHM_LOAD_FORMAT] is S.FlexTensorSharedLoader
