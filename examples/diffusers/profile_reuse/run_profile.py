"""Profile once, save the plans: ``python run_profile.py --out profiles/wan`` (needs diffusers)."""

import argparse

import torch

import flextensor_b200 as ft
from flextensor_b200.contrib.diffusers import WAN_INCLUDE_PATTERNS, offload_pipeline, save_pipeline_profiles


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="Wan-AI/Wan2.2-T2V-A14B-Diffusers")
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    from diffusers import WanPipeline

    pipe = WanPipeline.from_pretrained(args.model, torch_dtype=torch.bfloat16)
    offload_pipeline(pipe, ft.OffloadConfig(profiling_iters=20, include_patterns=WAN_INCLUDE_PATTERNS))
    pipe(prompt="warm-up", num_frames=81)
    save_pipeline_profiles(pipe, args.out)


if __name__ == "__main__":
    main()
