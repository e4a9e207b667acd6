"""Compiled offload with diffusers (needs diffusers).

``--mode per_unit``: each offload unit is compiled separately (``compile_fn``); the trap
boundaries stay in Python between compiled units.
``--mode external``: compile the whole transformer after offloading, with
``external_compile=True`` -- trap boundaries become the opaque custom ops
``flextensor_b200::pre_compute`` / ``post_compute`` inside the compiled graph.
"""

import argparse

import torch

import flextensor_b200 as ft
from flextensor_b200.contrib.diffusers import WAN_INCLUDE_PATTERNS, offload_pipeline


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="Wan-AI/Wan2.2-T2V-A14B-Diffusers")
    ap.add_argument("--mode", choices=["per_unit", "external"], default="per_unit")
    args = ap.parse_args()
    from diffusers import WanPipeline

    pipe = WanPipeline.from_pretrained(args.model, torch_dtype=torch.bfloat16)
    if args.mode == "per_unit":
        offload_pipeline(pipe, ft.OffloadConfig(include_patterns=WAN_INCLUDE_PATTERNS),
                         compile_fn=lambda unit: torch.compile(unit))
    else:
        offload_pipeline(pipe, ft.OffloadConfig(include_patterns=WAN_INCLUDE_PATTERNS, external_compile=True))
        pipe(prompt="warm-up", num_frames=81)  # discovery + profiling run eagerly
        pipe.transformer.compile()
        pipe.transformer_2.compile()
    pipe(prompt="A cat walks on the grass", num_frames=81)


if __name__ == "__main__":
    main()
