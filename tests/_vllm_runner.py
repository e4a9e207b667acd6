"""Subprocess body for the vLLM integration test: builds an engine on the given checkpoint and
prints the greedy continuation token ids of fixed prompts as one JSON line."""

import json
import sys


def main():
    path, worker = sys.argv[1], sys.argv[2]
    from vllm import LLM, SamplingParams

    kw = dict(model=path, skip_tokenizer_init=True, enforce_eager=True, gpu_memory_utilization=0.2,
              max_model_len=256, dtype="bfloat16", seed=0)
    if worker != "default":
        kw["worker_cls"] = worker
    if len(sys.argv) > 3:
        kw["load_format"] = sys.argv[3]
    llm = LLM(**kw)
    prompts = [{"prompt_token_ids": [(7 * i + 3 * j) % 2000 + 10 for j in range(24)]} for i in range(3)]
    outs = llm.generate(prompts, SamplingParams(max_tokens=16, temperature=0.0, detokenize=False))
    ids = [list(o.outputs[0].token_ids) for o in outs]
    extra = {}
    if worker != "default":
        import flextensor_b200 as ft

        try:
            om = ft.get_offload_manager("vllm")
            extra = {"phase": str(om.phase.value) if om.phase else None}
            tm = om.get_tensor_manager()
            extra["streamed_labels"] = sorted(tm.loader.plan.host_blocks) if tm and tm.loader else []
        except Exception as e:  # noqa: BLE001 - engine core may run in another process
            extra = {"note": f"manager not visible in this process: {e}"}
    print("RESULT " + json.dumps({"ids": ids, **extra}), flush=True)


if __name__ == "__main__":
    main()
