"""Wan2.2 T2V A14B through diffusers with both transformers' weights streamed from host memory.

    python examples/diffusers/quickstart/wan_t2v.py [--model Wan-AI/Wan2.2-T2V-A14B-Diffusers]

Needs ``diffusers`` and the checkpoint. The first pipeline call runs the discovery and
profiling passes; later calls run with the learned prefetch schedule.
"""

import argparse

import torch

import flextensor_b200 as ft
from flextensor_b200.contrib.diffusers import WAN_INCLUDE_PATTERNS, offload_pipeline, release_pipeline


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="Wan-AI/Wan2.2-T2V-A14B-Diffusers")
    ap.add_argument("--frames", type=int, default=81)
    ap.add_argument("--budget", type=float, default=None, help="max_gpu_mem_fraction (memory mode)")
    args = ap.parse_args()
    from diffusers import WanPipeline
    from diffusers.utils import export_to_video

    pipe = WanPipeline.from_pretrained(args.model, torch_dtype=torch.bfloat16)
    cfg = ft.OffloadConfig(profiling_iters=20, min_blocks=2, include_patterns=WAN_INCLUDE_PATTERNS,
                           max_gpu_mem_fraction=args.budget)
    offload_pipeline(pipe, cfg)
    prompt = "A cat walks on the grass, realistic"
    pipe(prompt=prompt, num_frames=args.frames)                    # discovery + profiling
    frames = pipe(prompt=prompt, num_frames=args.frames).frames[0]  # planned streaming
    export_to_video(frames, "wan-t2v.mp4", fps=16)
    release_pipeline(pipe)


if __name__ == "__main__":
    main()
