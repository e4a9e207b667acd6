"""Pipeline parallelism for the Wan DiT: the transformer blocks split into contiguous stages, one
per rank, with micro-batches (classifier-free-guidance halves, several prompts or videos)
flowing through them.

Stage 0 also runs the patch embedding, the last stage the output head. Every stage computes
the time and text conditioning itself from the (small) timestep and context inputs, so the
token activations ``[B, tokens, dim]`` are the only tensors that cross ranks.
:class:`~flextensor_b200.parallel.pp.PipelineStage` overlaps those transfers with the blocks.
The stages are balanced by the blocks' parameter bytes unless measured costs are given.

The reference has no pipeline parallelism (its shared-memory path requires PP = 1,
``src/flextensor/contrib/vllm/v2/worker.py:112-113``). Each stage's blocks form one module,
:class:`WanStageBlocks`, which :meth:`WanPipelineParallel.offload` hands to an offload manager
of its own (``wan_pp<stage>``), like the reference's per-denoiser managers; every micro-batch
is then one iteration of that manager.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

from flextensor_b200.models.wan import WanDiT
from flextensor_b200.parallel.pp import PipelineGroups, PipelineStage, TorchP2P, pipeline_groups, split_stages


def block_costs(model: WanDiT) -> list[float]:
    """Parameter bytes of every block: the default stage balance."""
    return [float(sum(p.numel() * p.element_size() for p in b.parameters())) for b in model.blocks]


class WanStageBlocks(nn.Module):
    """One stage's contiguous run of Wan blocks: the module an offload manager wraps."""

    def __init__(self, blocks: nn.ModuleList):
        super().__init__()
        self.blocks = blocks

    def forward(self, x, ctx, e, cos, sin):
        for blk in self.blocks:
            x = blk(x, ctx, e, cos, sin)
        return x


class WanPipelineParallel:
    """Keeps only this rank's stage of ``model.blocks`` (in place) and runs micro-batches
    through the pipeline. A collective constructor: every rank of ``group`` builds one."""

    def __init__(self, model: WanDiT, group=None, depth: int = 2, costs: Sequence[float] | None = None,
                 groups: PipelineGroups | None = None):
        self.groups = groups if groups is not None else pipeline_groups(group)
        self.n_stages = len(self.groups.ranks)
        self.stage = self.groups.ranks.index(dist.get_rank())
        self.bounds = split_stages(list(costs) if costs is not None else block_costs(model), self.n_stages)
        b0, b1 = self.bounds[self.stage]
        model.blocks = nn.ModuleList(list(model.blocks)[b0:b1])
        self.model = model
        self.stage_blocks: nn.Module = WanStageBlocks(model.blocks)
        self.depth = depth
        self.comm = TorchP2P(self.groups) if self.n_stages > 1 else None

    @torch.no_grad()
    def forward(self, latents: Sequence[torch.Tensor], timesteps: Sequence[torch.Tensor],
                contexts: Sequence[torch.Tensor]) -> list[torch.Tensor] | None:
        """Denoiser outputs for each micro-batch ``latents[i]`` ``[B_i, C, F, H, W]``, returned on
        the first and the last stage (None elsewhere). Stages other than the first read only the
        latents' shapes (meta tensors will do)."""
        m = self.model
        cfg = m.cfg
        dt = m.patch_embedding.weight.dtype
        device = m.patch_embedding.weight.device
        pf, ph, pw = cfg.patch
        grids = [(lat.shape[2] // pf, lat.shape[3] // ph, lat.shape[4] // pw) for lat in latents]
        tokens = [g[0] * g[1] * g[2] for g in grids]
        out_dim = m.proj_out.weight.shape[0]
        first, last = self.stage == 0, self.stage == self.n_stages - 1

        def fn(x: torch.Tensor, i: int) -> torch.Tensor:
            temb, e, ctx = m.condition(timesteps[i].to(device), contexts[i].to(device))
            if first:
                x, _ = m.patchify(x.to(device=device, dtype=dt))
                x = m._lin(x, m.patch_embedding, "bias").contiguous()
            cos, sin = m.rope(grids[i], device)
            x = self.stage_blocks(x, ctx, e, cos, sin)
            return m.head(x, temb) if last else x

        stage = PipelineStage(fn, self.stage, self.n_stages, self.comm, self.depth, device)
        outs = stage.run(len(latents), inputs=latents if first else None,
                         recv_spec=lambda i: ((latents[i].shape[0], tokens[i], cfg.dim), dt),
                         out_spec=lambda i: ((latents[i].shape[0], tokens[i], out_dim), dt))
        if outs is None:
            return None
        return [m.unpatchify(y, g) for y, g in zip(outs, grids)]

    __call__ = forward

    def offload(self, config, name: str | None = None) -> nn.Module:
        """Stream this stage's block weights under their own offload manager (default name
        ``wan_pp<stage>``); returns the manager's model proxy, which the pipeline then runs."""
        import flextensor_b200 as ft

        self.stage_blocks = ft.offload(self.stage_blocks, config, name=name or f"wan_pp{self.stage}")
        return self.stage_blocks
