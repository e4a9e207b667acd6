"""Serve with saved plans (no discovery/profiling): ``python run_infer.py --profiles profiles/wan``."""

import argparse

import torch

import flextensor_b200 as ft
from flextensor_b200.contrib.diffusers import WAN_INCLUDE_PATTERNS, offload_pipeline_from_profiles


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="Wan-AI/Wan2.2-T2V-A14B-Diffusers")
    ap.add_argument("--profiles", required=True)
    args = ap.parse_args()
    from diffusers import WanPipeline
    from diffusers.utils import export_to_video

    pipe = WanPipeline.from_pretrained(args.model, torch_dtype=torch.bfloat16)
    offload_pipeline_from_profiles(pipe, args.profiles, ft.OffloadConfig(include_patterns=WAN_INCLUDE_PATTERNS))
    export_to_video(pipe(prompt="A cat walks on the grass", num_frames=81).frames[0], "wan-t2v.mp4", fps=16)


if __name__ == "__main__":
    main()
