"""Pipeline parallelism of HLRT over the Tier-1 trunk (an extension: the
reference has no pipeline parallelism).

The trunk's blocks are split into ``num_stages`` contiguous ranges over the
ranks of a pipeline group.  Stage 0 also owns the embeddings; the last stage
owns everything after the trunk (gates, Tiers 2/3, conditioning, head and the
loss).  Activations ``(B, S, d)`` go forward and their gradients backward with
point-to-point ``isend``/``irecv`` (NCCL on GPUs, gloo on CPU); sends are
asynchronous, so a stage goes on with its next micro-batch while its output
travels, and waits for all of them at the end of the step.

:class:`PipelineStage` holds the stage's part of the model; :meth:`train_step`
runs one optimizer step's micro-batches with the one-forward-one-backward
schedule (``num_stages - stage - 1`` warm-up forwards, then alternating, then
cool-down backwards), so a stage keeps at most ``num_stages`` micro-batches of
activations alive.  Parameters outside the stage are dropped from it: each rank
stores and steps only its own.  The loss returned on the last stage is the mean
over micro-batches (gradients are scaled the same way), so one step equals the
unpipelined step on the concatenated batch.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn


def stage_ranges(num_layers: int, num_stages: int) -> List[tuple]:
    """Contiguous block ranges, the first stages one block longer when it does not divide."""
    base, extra = divmod(num_layers, num_stages)
    out, start = [], 0
    for s in range(num_stages):
        n = base + (1 if s < extra else 0)
        out.append((start, start + n))
        start += n
    return out


class PipelineStage(nn.Module):
    def __init__(self, model: nn.Module, group: Optional[dist.ProcessGroup] = None) -> None:
        super().__init__()
        self.model = model
        self.group = group
        self.num_stages = dist.get_world_size(group)
        self.stage = dist.get_rank(group)
        self.ranks = [dist.get_global_rank(group, i) if group is not None else i for i in range(self.num_stages)]
        L = len(model.tier1.layers)
        assert L >= self.num_stages, "need at least one Tier-1 block per stage"
        self.layer_range = stage_ranges(L, self.num_stages)[self.stage]
        self.first = self.stage == 0
        self.last = self.stage == self.num_stages - 1
        # a tied head: the first and the last stage both hold the embedding and add their
        # gradients (every rank creates the pair group, in the same order)
        self.tied = getattr(model, "output_proj", None) is None and self.num_stages > 1
        self.tie_group = dist.new_group([self.ranks[0], self.ranks[-1]]) if self.tied else None
        self._drop_foreign_parameters()

    # ------------------------------------------------------------ ownership
    def _owned(self, name: str) -> bool:
        if name.startswith("tier1.layers."):
            i = int(name.split(".")[2])
            return self.layer_range[0] <= i < self.layer_range[1]
        if name.startswith("tier1.memory_layers."):
            i = int(name.split(".")[2])
            return self.layer_range[0] <= i < self.layer_range[1]
        if name.startswith("embeddings."):
            tied = getattr(self.model, "output_proj", None) is None
            return self.first or (self.last and tied)  # the tied head reads the embedding on the last stage
        if name.startswith("tier1."):
            return True  # rotary tables
        return self.last

    def _drop_foreign_parameters(self) -> None:
        self.owned_names = [n for n, _ in self.model.named_parameters() if self._owned(n)]
        for name, p in list(self.model.named_parameters()):
            if not self._owned(name):
                p.requires_grad_(False)
                p.data = torch.empty(0, dtype=p.dtype, device=p.device)

    def sync_tied_gradients(self) -> None:
        """Sum the embedding gradient of the first and the last stage (call after
        :meth:`train_step`, before the optimizer step)."""
        if self.tied and (self.first or self.last):
            g = self.model.embeddings.weight.grad
            if g is None:
                g = torch.zeros_like(self.model.embeddings.weight)
                self.model.embeddings.weight.grad = g
            dist.all_reduce(g, group=self.tie_group)

    def stage_parameters(self) -> List[nn.Parameter]:
        named = dict(self.model.named_parameters())
        return [named[n] for n in self.owned_names]

    # ------------------------------------------------------------ compute
    def _forward(self, x: torch.Tensor) -> torch.Tensor:
        m = self.model
        h = m.embeddings(x) if self.first else x
        return m.tier1(h, layer_range=self.layer_range)

    def _send(self, t: torch.Tensor, to_stage: int):
        t = t.contiguous()
        return dist.isend(t, self.ranks[to_stage], group=self.group), t  # keep the buffer alive

    def _recv(self, shape, dtype, device, from_stage: int):
        buf = torch.empty(shape, dtype=dtype, device=device)
        return buf, dist.irecv(buf, self.ranks[from_stage], group=self.group)

    def train_step(self, micro_batches: Sequence[torch.Tensor], loss_fn: Callable[[dict, torch.Tensor], torch.Tensor],
                   act_shape, act_dtype: torch.dtype) -> Optional[torch.Tensor]:
        """Forward and backward of every micro-batch (1F1B).  ``micro_batches``: token ids
        (needed on the first stage for the embedding and on the last for the loss);
        ``loss_fn(outputs_after_tier1, ids) -> scalar`` on the last stage; ``act_shape``:
        the trunk activation shape of one micro-batch.  Returns the mean loss on the
        last stage, ``None`` elsewhere; gradients accumulate in the stage's parameters."""
        n = len(micro_batches)
        device = next(iter(self.stage_parameters()), torch.empty(0)).device
        warm = min(self.num_stages - self.stage - 1, n)
        inputs: List[Optional[torch.Tensor]] = [None] * n
        outputs: List[Optional[torch.Tensor]] = [None] * n
        pending = []
        losses = []

        def fwd(i: int) -> None:
            if self.first:
                x_in = micro_batches[i].to(device)
            else:
                x_in, req = self._recv(act_shape, act_dtype, device, self.stage - 1)
                req.wait()
                x_in.requires_grad_()
            inputs[i] = x_in
            out = self._forward(x_in)
            if self.last:
                loss = loss_fn(self.model.forward_after_tier1(out), micro_batches[i].to(device)) / n
                losses.append(loss.detach())
                outputs[i] = loss
            else:
                pending.append(self._send(out.detach(), self.stage + 1))
                outputs[i] = out

        def bwd(i: int) -> None:
            if self.last:
                outputs[i].backward()
            else:
                g, req = self._recv(act_shape, act_dtype, device, self.stage + 1)
                req.wait()
                torch.autograd.backward(outputs[i], g)
            if not self.first:
                pending.append(self._send(inputs[i].grad, self.stage - 1))
            inputs[i] = outputs[i] = None

        for i in range(warm):
            fwd(i)
        b = 0
        for i in range(warm, n):
            fwd(i)
            bwd(b)
            b += 1
        while b < n:
            bwd(b)
            b += 1
        for work, _ in pending:
            work.wait()
        return torch.stack(losses).sum() if self.last else None


def _bench(argv=None) -> None:
    """``torchrun --nproc-per-node P -m llm_research_b200.parallel.pipeline``: time the
    1F1B forward + backward of one step (``--micro-batches`` of ``--micro x --seq``
    tokens) of a preset on P GPUs, one stage per GPU, with CUDA events (max over
    ranks; the optimizer step is not part of it); rank 0 prints a JSON line."""
    import argparse
    import datetime
    import json
    import os

    import torch.nn.functional as F

    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config

    ap = argparse.ArgumentParser(description=_bench.__doc__.split("\n")[0])
    ap.add_argument("--preset", default="genesis-1b")
    ap.add_argument("--micro-batches", type=int, default=8)
    ap.add_argument("--micro", type=int, default=1)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    cfg = build_hlrt_config(args.preset)
    torch.manual_seed(0)
    with torch.device(device):
        model = HLRT(cfg).to(torch.bfloat16)
    st = PipelineStage(model)
    g = torch.Generator().manual_seed(1)
    mbs = [torch.randint(0, cfg.vocab_size, (args.micro, args.seq), generator=g) for _ in range(args.micro_batches)]

    def loss_fn(out, ids):
        logits = out["logits"]
        return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1))

    def step():
        for p in st.stage_parameters():
            p.grad = None
        st.train_step(mbs, loss_fn, act_shape=(args.micro, args.seq, cfg.d_model), act_dtype=torch.bfloat16)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = torch.tensor([start.elapsed_time(end) / args.steps], device=device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    tokens = args.micro_batches * args.micro * args.seq
    if dist.get_rank() == 0:
        print(json.dumps({"case": "pipeline_1f1b", "preset": args.preset, "stages": dist.get_world_size(),
                          "micro_batches": args.micro_batches, "tokens_per_step": tokens,
                          "ms_per_step": ms.item(), "tokens_per_s": tokens / (ms.item() / 1e3),
                          "note": "forward + backward of one step, no optimizer"}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench()
