"""Pipeline parallelism: a model's blocks split into contiguous stages over the ranks of one node,
micro-batches flowing stage 0 -> 1 -> ... -> N-1 over NCCL point-to-point, overlapped with compute.

The reference has no pipeline parallelism: its shared-memory path requires PP = 1
(``src/flextensor/contrib/vllm/v2/worker.py:112-113``) and only its shared-memory namespaces carry
a ``_pp{r}`` rank suffix (``src/flextensor/shm/namespace.py:76-96``). Here the activations
between stages are the only data that crosses ranks, and they go over NCCL send/recv, not over
kernels of this package: a stage boundary moves one activation per micro-batch between two
GPUs, with no compute to fuse it into.

Overlap. A stage posts the receive of micro-batch ``m + depth`` as soon as it has taken
micro-batch ``m``, so up to ``depth`` receives are in flight while it computes. Its send of
``m``'s output is posted right after the compute, and runs while it computes ``m + 1``. Three
communicators keep the transfers from queueing behind one another:

* the links (r, r+1) alternate between two groups by the parity of r, so a rank receives from
  its predecessor and sends to its successor on different communicators (and, with NCCL,
  different internal streams): a send that waits for its receiver never holds up the receive
  of the next micro-batch;
* outputs that go back from the last stage to the first use a third group, so that a first
  stage still sending inputs is never blocked by a pending return. The first stage posts all
  its return receives up front, and the last stage sends each output back as soon as it is
  computed.

With NCCL, ``isend`` / ``irecv`` enqueue on NCCL's own streams and ``wait()`` only orders the
current CUDA stream after the transfer, so the host runs ahead and the GPU overlaps the
transfers with the stage's kernels.

A sequence of denoising steps cannot be pipelined across steps (step t+1 needs step t's
output); the micro-batches of one step (classifier-free guidance halves, several prompts or
videos) fill the pipeline.
"""

from __future__ import annotations

from collections import deque
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any, Protocol, runtime_checkable

import torch
import torch.distributed as dist

__all__ = ["PipelineGroups", "PipelineStage", "TorchP2P", "connect_pipeline", "pipeline_groups", "split_stages"]


def split_stages(costs: Sequence[float], n_stages: int) -> list[tuple[int, int]]:
    """Split items with the given costs into ``n_stages`` contiguous ``[start, end)`` ranges
    that minimise the largest stage's total cost (exact linear-partition dynamic programme;
    ties keep the earlier boundary). Every stage gets at least one item."""
    n = len(costs)
    if n_stages < 1 or n < n_stages:
        raise ValueError(f"cannot split {n} items into {n_stages} non-empty stages")
    if any(c < 0 for c in costs):
        raise ValueError("stage costs must be non-negative")
    prefix = [0.0]
    for c in costs:
        prefix.append(prefix[-1] + float(c))
    inf = float("inf")
    # best[k][i]: smallest possible max-stage cost of the first i items split into k stages
    best = [[inf] * (n + 1) for _ in range(n_stages + 1)]
    cut = [[0] * (n + 1) for _ in range(n_stages + 1)]
    best[0][0] = 0.0
    for k in range(1, n_stages + 1):
        for i in range(k, n - (n_stages - k) + 1):
            for j in range(k - 1, i):
                v = max(best[k - 1][j], prefix[i] - prefix[j])
                if v < best[k][i]:
                    best[k][i], cut[k][i] = v, j
    bounds = []
    i = n
    for k in range(n_stages, 0, -1):
        j = cut[k][i]
        bounds.append((j, i))
        i = j
    return bounds[::-1]


@dataclass
class PipelineGroups:
    """The communicators of one pipeline: ``links[r % 2]`` carries the link from stage r to
    stage r+1, ``back`` carries outputs from the last stage to the first. ``ranks[s]`` is the
    global rank of stage s."""

    ranks: list[int]
    links: tuple[Any, Any]
    back: Any


def pipeline_groups(group: Any = None) -> PipelineGroups:
    """Create the pipeline's communicators over ``group``'s ranks, in group-rank order. A
    collective call: every process of the default group calls it (``new_group`` needs them all)."""
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    even, odd, back = (dist.new_group(ranks) for _ in range(3))
    groups = PipelineGroups(ranks=ranks, links=(even, odd), back=back)
    if dist.get_rank() in ranks and len(ranks) > 1:
        connect_pipeline(groups)
    return groups


def connect_pipeline(groups: PipelineGroups) -> None:
    """Open every point-to-point connection the pipeline uses, on every rank in the same order.

    NCCL opens the connection between two ranks of a communicator at their first send/receive
    pair, and that handshake blocks the host until the peer reaches the same communicator. A
    pipeline's first operations differ by stage (the first stage posts its return receives on
    ``back``, the second its forward receives on ``links[0]``), so without this each could wait
    for the other. Here each communicator in turn exchanges one element with both ring
    neighbours (stage s with s - 1 and s + 1, which covers every link and the last-to-first
    return) as one batched group."""
    me = groups.ranks.index(dist.get_rank())
    n = len(groups.ranks)
    nxt, prv = groups.ranks[(me + 1) % n], groups.ranks[(me - 1) % n]
    backend = dist.get_backend(groups.back)
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    for g in (groups.links[0], groups.links[1], groups.back):
        out = torch.zeros(2, device=device)
        inp = torch.empty(2, device=device)
        ops = [dist.P2POp(dist.isend, out[0:1], nxt, g), dist.P2POp(dist.irecv, inp[0:1], prv, g),
               dist.P2POp(dist.isend, out[1:2], prv, g), dist.P2POp(dist.irecv, inp[1:2], nxt, g)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@runtime_checkable
class Handle(Protocol):
    def wait(self) -> Any: ...


@runtime_checkable
class P2P(Protocol):
    """Point-to-point transport between pipeline stages. ``channel`` is ``"fwd"`` for the
    stage-to-stage link and ``"back"`` for the last-to-first return."""

    def send(self, t: torch.Tensor, src_stage: int, dst_stage: int, channel: str) -> Handle: ...

    def recv(self, t: torch.Tensor, src_stage: int, dst_stage: int, channel: str) -> Handle: ...


class TorchP2P:
    """:class:`P2P` over ``torch.distributed`` (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, groups: PipelineGroups):
        self.g = groups

    def _group(self, src_stage: int, channel: str):
        return self.g.back if channel == "back" else self.g.links[src_stage % 2]

    def send(self, t, src_stage, dst_stage, channel):
        return dist.isend(t, dst=self.g.ranks[dst_stage], group=self._group(src_stage, channel))

    def recv(self, t, src_stage, dst_stage, channel):
        return dist.irecv(t, src=self.g.ranks[src_stage], group=self._group(src_stage, channel))


Spec = tuple[Sequence[int], torch.dtype]


class PipelineStage:
    """One rank's stage of a pipeline.

    ``fn(x, m)`` computes micro-batch ``m`` on this stage: on the first stage ``x`` is the
    caller's input ``m``; on the others it is the previous stage's output, received into a
    buffer of ``recv_spec(m) = (shape, dtype)``. ``depth`` bounds the receives posted ahead.
    """

    def __init__(self, fn: Callable[[torch.Tensor, int], torch.Tensor], stage: int, n_stages: int,
                 comm: P2P | None = None, depth: int = 2, device: torch.device | str | None = None):
        if not 0 <= stage < n_stages:
            raise ValueError(f"stage {stage} outside 0..{n_stages - 1}")
        if depth < 1:
            raise ValueError("depth must be at least 1")
        if n_stages > 1 and comm is None:
            raise ValueError("a pipeline of several stages needs a transport")
        self.fn, self.stage, self.n_stages, self.comm, self.depth = fn, stage, n_stages, comm, depth
        self.device = torch.device(device) if device is not None else None

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.n_stages - 1

    def _buffer(self, spec: Spec) -> torch.Tensor:
        shape, dtype = spec
        return torch.empty(tuple(shape), dtype=dtype, device=self.device)

    def run(self, n_micro: int, inputs: Sequence[torch.Tensor] | None = None,
            recv_spec: Callable[[int], Spec] | None = None, out_spec: Callable[[int], Spec] | None = None
            ) -> list[torch.Tensor] | None:
        """Run ``n_micro`` micro-batches through this stage.

        The last stage returns its outputs. With ``out_spec`` given, they also go back to the
        first stage, which returns them too; every other stage returns None. ``inputs`` is
        read on the first stage only, ``recv_spec`` on the others."""
        if self.is_first and (inputs is None or len(inputs) != n_micro):
            raise ValueError(f"the first stage needs {n_micro} inputs")
        if not self.is_first and recv_spec is None:
            raise ValueError("stages after the first need recv_spec to size their receives")
        s = self.stage
        pending: deque[tuple[torch.Tensor, Handle]] = deque()
        sends: list[tuple[Handle, torch.Tensor]] = []  # keeps every sent tensor alive until done

        def post(m: int) -> None:
            buf = self._buffer(recv_spec(m))
            pending.append((buf, self.comm.recv(buf, s - 1, s, "fwd")))

        returning = out_spec is not None and self.n_stages > 1
        back: list[tuple[torch.Tensor, Handle]] = []
        if returning and self.is_first:  # the return path has its own communicator: post it all now
            for m in range(n_micro):
                buf = self._buffer(out_spec(m))
                back.append((buf, self.comm.recv(buf, self.n_stages - 1, 0, "back")))
        if not self.is_first:
            for m in range(min(self.depth, n_micro)):
                post(m)
        outs: list[torch.Tensor] = []
        for m in range(n_micro):
            if self.is_first:
                x = inputs[m]
            else:
                x, h = pending.popleft()
                h.wait()
                if m + self.depth < n_micro:
                    post(m + self.depth)
            y = self.fn(x, m)
            if self.is_last:
                outs.append(y)
                if returning:  # each output heads back while the next micro-batch computes
                    y = y.contiguous()
                    sends.append((self.comm.send(y, s, 0, "back"), y))
            else:
                y = y.contiguous()
                sends.append((self.comm.send(y, s, s + 1, "fwd"), y))
        result: list[torch.Tensor] | None = outs if self.is_last else None
        if back:
            for _, h in back:
                h.wait()
            result = [buf for buf, _ in back]
        for h, _ in sends:
            h.wait()
        return result
