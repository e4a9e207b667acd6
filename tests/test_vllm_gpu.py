"""vLLM integration: a tiny random-init Llama served by vLLM with the FlexTensor worker must
produce the same greedy tokens as vLLM's own worker (weights stream from host memory; the
math is vLLM's in both runs)."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _have_vllm():
    try:
        import vllm  # noqa: F401

        return True
    except Exception:  # noqa: BLE001
        return False


@pytest.fixture(scope="module")
def tiny_llama(tmp_path_factory):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    d = tmp_path_factory.mktemp("tiny_llama")
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1536, num_hidden_layers=6,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=512,
                      rope_theta=500000.0, torch_dtype="bfloat16", tie_word_embeddings=False)
    torch.manual_seed(0)
    m = LlamaForCausalLM(cfg).to(torch.bfloat16)
    m.save_pretrained(str(d), safe_serialization=True)
    return str(d)


_BASE: dict = {}


def _base_ids(path):
    if path not in _BASE:
        _BASE[path] = _run(path, "default")["ids"]
    return _BASE[path]


def _run(path, worker, extra_env=None, load_format=None):
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    env["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    env.update(extra_env or {})
    args = [sys.executable, os.path.join(ROOT, "tests", "_vllm_runner.py"), path, worker]
    if load_format:
        args.append(load_format)
    p = subprocess.run(args, capture_output=True, text=True, env=env, timeout=600)
    line = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")]
    assert p.returncode == 0 and line, f"vLLM run failed ({worker}):\n{p.stdout[-3000:]}\n{p.stderr[-6000:]}"
    return json.loads(line[-1][len("RESULT "):])


@pytest.mark.skipif(not _have_vllm(), reason="vllm not installed")
def test_vllm_worker_streams_and_matches(tiny_llama):
    base = {"ids": _base_ids(tiny_llama)}
    ft_env = {"FT_ENABLED": "1", "FT_MAX_GPU_MEM_FRACTION": "0.00008", "FT_NUM_BLOCKS": "2",
              "FT_MIN_BLOCKS": "2"}
    ours = _run(tiny_llama, "flextensor_b200.contrib.vllm.worker.FlexTensorOffloadWorker", ft_env)
    assert ours.get("phase") == "inference", ours
    assert ours.get("streamed_labels"), f"nothing was streamed: {ours}"
    assert ours["ids"] == base["ids"]


@pytest.mark.skipif(not _have_vllm(), reason="vllm not installed")
def test_vllm_host_first_loader_matches(tiny_llama):
    """``load_format="flextensor"``: the model is built and loaded on the host, post-load
    processing runs per unit on the GPU, and (FlexTensor disabled) the model then moves to the
    GPU; the greedy tokens match vLLM's own loader."""
    ours = _run(tiny_llama, "flextensor_b200.contrib.vllm.worker.FlexTensorOffloadWorker", {"FT_ENABLED": "0"},
                load_format="flextensor")
    assert ours["ids"] == _base_ids(tiny_llama)
