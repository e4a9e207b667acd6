"""vLLM with tensor parallelism 2: the FlexTensor worker's fused GEMM + all-reduce on the
row-parallel layers (FT_VLLM_FUSED_TP=1) must generate the same greedy tokens as vLLM's own
all-reduce for a tiny random-init Llama (and run with weight offloading on as well)."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu, pytest.mark.slow]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA devices", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def tiny_llama(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM

    d = tmp_path_factory.mktemp("tiny_llama_tp")
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1536, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=512,
                      torch_dtype="bfloat16", tie_word_embeddings=False)
    torch.manual_seed(0)
    LlamaForCausalLM(cfg).to(torch.bfloat16).save_pretrained(str(d), safe_serialization=True)
    return str(d)


def _run(path, env_extra):
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), NCCL_NVLS_ENABLE="0")
    env.update(env_extra)
    code = f"""
import json
from vllm import LLM, SamplingParams
llm = LLM(model={path!r}, skip_tokenizer_init=True, enforce_eager=True, tensor_parallel_size=2,
          gpu_memory_utilization=0.2, max_model_len=256, dtype="bfloat16", seed=0,
          worker_cls="flextensor_b200.contrib.vllm.worker.FlexTensorOffloadWorker",
          disable_custom_all_reduce=True)
prompts = [{{"prompt_token_ids": [(5 * i + 3 * j) % 2000 + 10 for j in range(20)]}} for i in range(3)]
outs = llm.generate(prompts, SamplingParams(max_tokens=8, temperature=0.0, detokenize=False))
print("RESULT " + json.dumps([list(o.outputs[0].token_ids) for o in outs]), flush=True)
"""
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    line = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")]
    assert p.returncode == 0 and line, f"vLLM TP=2 run failed:\n{p.stdout[-2000:]}\n{p.stderr[-6000:]}"
    return json.loads(line[-1][len("RESULT "):])


def test_fused_tp_allreduce_matches_vllm(tiny_llama):
    base = _run(tiny_llama, {"FT_VLLM_FUSED_TP": "0"})
    fused = _run(tiny_llama, {"FT_VLLM_FUSED_TP": "1"})
    same = sum(a[:2] == b[:2] for a, b in zip(base, fused))
    assert same == len(base), f"first tokens differ: {base} vs {fused}"
    offl = _run(tiny_llama, {"FT_VLLM_FUSED_TP": "1", "FT_ENABLED": "1", "FT_MAX_GPU_MEM_FRACTION": "0.00004"})
    assert [o[:2] for o in offl] == [o[:2] for o in base]
