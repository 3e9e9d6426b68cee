#!/usr/bin/env python
"""Training-throughput benchmark: GENESIS-1B dense (24 layers, d_model 2048,
16 heads, SwiGLU ffn 5632, vocab 32000, RoPE), seq 4096, bf16, fully sharded
data parallel with distributed Muon, synthetic uniform token ids, random
N(0, 0.02) weights.

Weak scaling: every GPU processes 32 sequences per optimizer step (global
batch 256 at 8 GPUs), as micro-batches accumulated in fp32.

One step = all micro-batches of one optimizer step, including the gradient
reduce-scatter, clipping, the distributed Muon/AdamW update and the weight
refresh.  Two timed phases, each bracketed by barrier + synchronize:

* device-timed: inputs staged on the GPU beforehand; CUDA events on the
  launching stream; the reported ``value`` uses the max over ranks;
* end-to-end (``e2e``): the public trainer API called with inputs in pinned
  host memory (copied host->device inside the step) and the step's loss read
  back to the host every step; host wall clock, max over ranks.

Inputs and activations are far larger than the 126 MB L2 (no flush needed).

``--impl reference`` runs the unmodified reference installation in
``baseline/_ref`` through its own ``DistributedBootstrapTrainer`` on the same
configuration and prints the same JSON line with ``"impl": "reference"``.

Usage: ``python bench.py [--gpus N] [--steps K] [--warmup W]``; for N > 1 launch
one process per GPU with ``torch.distributed.run``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
METRIC = "train tokens/sec/box (device-timed, max over ranks) at 1/2/4/8 B200; exposed comm ms/step"
MODEL_NAME = "GENESIS-1B dense (HLRT trunk: 24L, d2048, 16H, SwiGLU 5632, vocab 32000, RoPE)"
MODEL_NAMES = {
    "genesis-1b": MODEL_NAME,
    "genesis-7b": "GENESIS-7B dense (32L, d4096, 32/8 heads, SwiGLU 11008, vocab 32000)",
    "genesis-7b-nvfp4": "GENESIS-7B dense NVFP4 (32L, d4096, 32/8 heads, SwiGLU 11008, vocab 32000)",
    "genesis-40b-moe": "GENESIS-40B-A8B MoE (32L, d4096, 32/8 heads, 16 experts x ffn 6144 top-2 + 1 shared)",
}


# HLRTConfig fields of the benchmarked model for the reference arm, written out
# here so that the reference process imports nothing from this repository.  The
# 24-layer dense trunk is Tier 1; tiers 2 and 3 carry no transformer layers.
REFERENCE_FIELDS = {
    "genesis-1b": dict(
        vocab_size=32000, d_model=2048,
        tier1_num_layers=24, tier1_num_heads=16, tier1_num_kv_heads=None, tier1_d_ff=5632, tier1_max_seq_len=4096,
        gate1_chunk_size=32, num_latent_vectors=8, latent_pool_num_heads=16,
        tier2_d_model=2048, tier2_num_layers=0, tier2_num_heads=16, tier2_max_seq_len=1024,
        tier3_d_model=2048, tier3_num_layers=0, tier3_num_heads=16, tier3_max_seq_len=1024,
        tier3_recurrence_steps=1,
    ),
}


_REASON_BITS = {
    "applications_clocks_setting": 0x2,
    "sw_power_cap": 0x4,
    "hw_slowdown": 0x8,
    "sync_boost": 0x10,
    "sw_thermal_slowdown": 0x20,
    "hw_thermal_slowdown": 0x40,
    "hw_power_brake_slowdown": 0x80,
    "display_clock_setting": 0x100,
}


class ClockSampler:
    """Read-only NVML sampling of SM clock, power and active clock-event reasons
    every ``period_s`` while the timed region runs (nothing is ever set).

    Defined here rather than imported so that the reference arm loads no module
    of this repository."""

    def __init__(self, device_index: int = 0, period_s: float = 0.2) -> None:
        import threading

        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._ok = False
        try:
            import pynvml  # nvidia_ml_py

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self._ok = True
        except Exception:
            self._ok = False

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                util = nv.nvmlDeviceGetUtilizationRates(self._h).gpu
                self.samples.append({"sm_mhz": float(sm), "power_w": pw, "util": float(util)})
                for name, bit in _REASON_BITS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        import threading

        if self._ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)

    def summary(self) -> dict:
        import statistics

        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        loaded = [x["sm_mhz"] for x in self.samples if x["util"] > 50] or [x["sm_mhz"] for x in self.samples]
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
            "power_w_max": max((x["power_w"] for x in self.samples), default=None),
        }


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--preset", default="genesis-1b")
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--per-gpu-seqs", type=int, default=32)
    ap.add_argument("--micro-batch", type=int, default=16)
    ap.add_argument("--ref-micro-batch", type=int, default=0,
                    help="reference micro-batch; 0 = 2 (the largest that fits its fp32 O(S^2) attention on one "
                         "B200 at seq 4096), then 1 if that runs out of memory on one GPU")
    ap.add_argument("--ref-e2e-steps", type=int, default=3,
                    help="end-to-end steps of the reference arm (its step takes tens of seconds)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--precision", choices=["bf16", "nvfp4"], default="bf16",
                    help="linear-layer precision of the model (nvfp4: block-scaled FP4 training GEMMs)")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel group size for the Tier-1 trunk (consecutive ranks); FSDP over the rest")
    ap.add_argument("--ep", action="store_true",
                    help="expert parallelism over all ranks for MoE presets (each rank holds E/world experts)")
    ap.add_argument("--fused-loss", action="store_true",
                    help="head + cross-entropy chunk by chunk without the full logits (vocabulary-parallel under --tp)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--count-launches", type=int, default=1)
    return ap.parse_args(argv)


def _max_over_ranks(x: float, dist, device) -> float:
    import torch

    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier_sync(dist, torch):
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def _count_kernels(step_fn, prefixes=("lrb::",)) -> int:
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if getattr(ev, "device_type", None) is not None and str(ev.device_type).endswith("CUDA"):
            if any(p in ev.name for p in prefixes):
                n += 1
    return n


def run_ours(args) -> dict:
    sys.path.insert(0, REPO)
    import torch
    import torch.distributed as dist

    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_distributed import DistributedBootstrapTrainer, init_distributed
    from llm_research_b200.models.presets import build_hlrt_config, count_flops_per_token
    from olympus.data.tokenizer import TokenizerWrapper
    from olympus.distributed.fsdp_wrapper import FSDPConfig

    local_rank, world, rank = init_distributed(timeout_s=300.0)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    micro = args.micro_batch
    accum = max(args.per_gpu_seqs // micro, 1)
    S = args.seq_len
    cfg = build_hlrt_config(args.preset)
    torch.manual_seed(args.seed)
    from llm_research_b200.ops.linear import set_linear_precision

    set_linear_precision(args.precision)
    import contextlib

    ep_ctx = contextlib.nullcontext()
    tp = args.tp
    assert world % tp == 0, "--tp must divide the number of GPUs"
    dp_world, dp_rank = world // tp, rank // tp
    tp_group = dp_group = tp_comm = None
    if tp > 1:
        from llm_research_b200.parallel.tp import TPComm, tensor_parallel

        for i in range(dp_world):  # every rank creates every group, in the same order
            grp = dist.new_group(list(range(i * tp, (i + 1) * tp)))
            if i == dp_rank:
                tp_group = grp
        for j in range(tp):
            grp = dist.new_group(list(range(j, world, tp)))
            if j == rank % tp:
                dp_group = grp
        d_ff = cfg.tier1_d_ff or 4 * cfg.d_model
        width = max(2 * d_ff // tp, (cfg.tier1_num_heads + 2 * (cfg.tier1_num_kv_heads or cfg.tier1_num_heads))
                    * (cfg.d_model // cfg.tier1_num_heads) // tp, cfg.d_model)
        tp_comm = TPComm(tp_group, max_tokens=micro * S, max_width=width, device=device)
        ep_ctx = tensor_parallel(tp_group, tp_comm)
    if args.ep and cfg.tier1_moe_num_experts:
        from llm_research_b200.parallel.expert_parallel import EPComm, expert_parallel

        comm = None
        if world > 1:
            comm = EPComm(None, max_tokens=micro * S, top_k=cfg.tier1_moe_top_k, d=cfg.d_model,
                          experts_per_rank=cfg.tier1_moe_num_experts // world,
                          capacity_factor=cfg.tier1_moe_capacity_factor, device=device)
        ep_ctx = expert_parallel(None, comm)
    with torch.device(device), ep_ctx:
        model = HLRT(cfg)
    trainer = DistributedBootstrapTrainer(
        model,
        optimizer_kwargs={"lr_muon": 0.02, "lr_adamw": 3e-4, "weight_decay_adamw": 0.01, "ns_steps": 5},
        scheduler_kwargs={"base_lr": 3e-4, "min_lr": 2e-5, "warmup_steps": 10, "total_steps": 1000},
        tokenizer=TokenizerWrapper(backend="char", vocab_size=cfg.vocab_size),
        config={"gradient_accumulation_steps": accum, "max_grad_norm": 1.0, "sync_metrics": False},
        fsdp_config=FSDPConfig(sharding_strategy="FULL_SHARD", mixed_precision="bf16", activation_checkpointing=False,
                               process_group=dp_group, tp_group=tp_group),
    )
    # A distinct batch for every step (warm-up, device-timed and end-to-end
    # phases draw from one pool in order), so the loss is a real cross-N check
    # rather than memorisation of one batch.  Ranks of one tensor-parallel group
    # train on the same sequences.
    g = torch.Generator().manual_seed(args.seed * 1000 + dp_rank)
    n_pool = args.warmup + args.steps
    host = torch.randint(0, cfg.vocab_size, (n_pool, accum, micro, S), generator=g, dtype=torch.int64).pin_memory()
    dev_pool = host.to(device)

    def step(batches):
        out = None
        for b in batches:
            out = trainer.train_step({"input_ids": b, "fused_lm_loss": args.fused_loss})
        return out["loss"]

    for i in range(args.warmup):
        step(dev_pool[i])
    _barrier_sync(dist, torch)

    sampler = ClockSampler(device_index=local_rank)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        _barrier_sync(dist, torch)
        e0.record()
        for i in range(args.steps):
            loss = step(dev_pool[args.warmup + i])
        e1.record()
        _barrier_sync(dist, torch)
    dev_ms = _max_over_ranks(e0.elapsed_time(e1), dist, device)
    final_loss = float(loss)
    del dev_pool

    e2e = None
    if not args.no_e2e:
        _barrier_sync(dist, torch)
        t0 = time.perf_counter()
        for i in range(args.steps):
            # pinned host batch, copied host -> device inside the step
            l = step(host[(args.warmup + i) % n_pool])
            lv = float(l)  # device -> host read of the step's result
        _barrier_sync(dist, torch)
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dist, device)
        e2e = {
            "value": dp_world * accum * micro * S * args.steps / e2e_s,
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(host[0].numel() * host.element_size()),
            "d2h_bytes_per_step": 4,
            "ms_per_step": e2e_s * 1000.0 / args.steps,
        }

    launches = None
    if args.count_launches:
        per_step = _count_kernels(lambda: step(host[0].to(device)))
        launches = per_step * args.steps

    # Exposed communication: one extra (untimed) step with the compute stream's
    # waits on communication events bracketed by CUDA events; max over ranks.
    exposed = None
    engine = trainer.model
    if world > 1 and hasattr(engine, "start_exposed_comm_measurement"):
        _barrier_sync(dist, torch)
        engine.start_exposed_comm_measurement()
        step(host[1 % n_pool].to(device))
        exposed = _max_over_ranks(engine.stop_exposed_comm_measurement(), dist, device)

    tokens_per_step = dp_world * accum * micro * S
    value = tokens_per_step * args.steps / (dev_ms / 1000.0)
    flops = count_flops_per_token(cfg, S)
    res = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform token ids, seeded); random N(0,0.02) init",
        "impl": "ours",
        "config": {
            "model": MODEL_NAMES.get(args.preset, args.preset),
            "global_batch": dp_world * accum * micro,
            "seq_len": S,
            "micro_batch": micro,
            "grad_accum": accum,
            "parallelism": (f"fsdp{dp_world} (FULL_SHARD, bf16 compute, fp32 master) + distributed Muon"
                            + (f" + tp{tp} (sequence parallel Tier 1)" if tp > 1 else "")
                            + (f" + ep{world}" if args.ep else "")),
            "linear_precision": args.precision,
            "loss": ("fused head + CE" + (" (vocabulary-parallel)" if tp > 1 else "")) if args.fused_loss else "logits + CE",
            "preset": args.preset,
            "optimizer": "MuonAdamWHybrid (Muon on 2-D, AdamW on embedding/norms)",
            "l2": "inputs+activations >> 126 MB L2; no flush",
            "model_tflops_per_gpu": flops * value / world / 1e12,
            "exposed_comm_ms_per_step": exposed,
            "comm": (getattr(trainer.model, "comm", "none") if dp_world > 1 else "none (one rank)"),
            "final_loss": final_loss,
        },
        "clocks": sampler.summary(),
        "e2e": e2e,
        "gpu_launches": launches,
    }
    if dist.is_initialized():
        dist.barrier()
        if tp_comm is not None:
            tp_comm.close()
        dist.destroy_process_group()
    return res if rank == 0 else None


def run_reference(args) -> dict:
    """The unmodified reference (installed into baseline/_ref) through its public API."""
    ref = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "genesis")) or not os.path.isdir(os.path.join(ref, "olympus")):
        return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
    # Make sure its packages, not this repository's, are imported.
    sys.path[:] = [p for p in sys.path if os.path.abspath(p or os.getcwd()) != REPO]
    sys.path.insert(0, ref)
    for mod in [m for m in list(sys.modules) if m.split(".")[0] in ("genesis", "olympus")]:
        del sys.modules[mod]
    import torch
    import torch.distributed as dist

    import genesis
    from genesis.model.hlrt import HLRT, HLRTConfig
    from genesis.training.train_phase1_distributed import DistributedBootstrapTrainer
    from olympus.data.tokenizer import TokenizerWrapper
    from olympus.optim.muon_adamw_hybrid import MuonAdamWHybrid
    from olympus.optim.schedulers import WSDScheduler

    assert os.path.abspath(genesis.__file__).startswith(ref), genesis.__file__
    if args.preset not in REFERENCE_FIELDS:
        return {"impl": "reference", "unavailable": f"no reference configuration for preset {args.preset}"}
    fields = dict(REFERENCE_FIELDS[args.preset])
    # The reference runs only in fp32: in bf16 its latent pooling multiplies by a
    # float mask (genesis/model/latent_pooling.py:171) and the tier-2 linear then
    # fails on mixed dtypes, and the installed flash-attn rejects fp32, so its
    # own vanilla attention path is selected through the config flags.
    fields.update(tier1_use_flash_attention=False, tier2_use_flash_attention=False, tier3_use_flash_attention=False)
    cfg = HLRTConfig(**fields)
    from olympus.distributed.fsdp_wrapper import FSDPConfig
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1 and not dist.is_initialized():
        # The reference joins an existing process group; a short timeout makes a rank
        # whose peer failed end with an error instead of waiting ten minutes.
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    S = args.seq_len
    if args.ref_micro_batch > 0:
        candidates = [args.ref_micro_batch]
    else:
        # 2 fits on a B200 (4 and 8 run out of memory); on several GPUs no fallback,
        # since a probe that runs out of memory on one rank would leave the others
        # in a collective
        candidates = [2, 1] if world == 1 else [2]

    def build(micro):
        torch.manual_seed(args.seed)
        model = HLRT(cfg)
        accum = max(args.per_gpu_seqs // micro, 1)
        trainer = DistributedBootstrapTrainer(
            # The reference's sharded strategies fail at world > 1: FULL_SHARD in the tied
            # output head, which reads embeddings.weight after its FSDP unit resharded it
            # ("size mismatch, got input (16384), mat (16384x2048), vec (32768000)");
            # SHARD_GRAD_OP in FSDP's gradient finalisation after its no_sync accumulation
            # ("All sharded parameters that received a gradient in the post-backward should
            # use `_saved_grad_shard`").  Its NO_SHARD strategy (replicated, DDP-like) runs.
            fsdp_config=FSDPConfig(sharding_strategy="NO_SHARD", mixed_precision="fp32",
                                   activation_checkpointing=True) if world > 1 else None,
            model=model,
            optimizer_cls=MuonAdamWHybrid,
            optimizer_kwargs={"lr_muon": 0.02, "lr_adamw": 3e-4, "weight_decay_adamw": 0.01, "ns_steps": 5},
            scheduler_cls=WSDScheduler,
            scheduler_kwargs={"base_lr": 3e-4, "min_lr": 2e-5, "warmup_steps": 10, "total_steps": 1000},
            tokenizer=TokenizerWrapper(backend="char"),
            config={"gradient_accumulation_steps": accum, "max_grad_norm": 1.0},
        )
        g = torch.Generator().manual_seed(args.seed * 1000 + rank)
        host = torch.randint(0, cfg.vocab_size, (accum, micro, S), generator=g, dtype=torch.int64).pin_memory()
        return trainer, accum, host

    trainer = None
    for i, micro in enumerate(candidates):
        try:
            trainer, accum, host = build(micro)
            for j in range(accum):  # one whole optimizer step as the fit probe (extra warm-up)
                trainer.train_step({"input_ids": host[j].to(device)})
            torch.cuda.synchronize()
            break
        except torch.OutOfMemoryError:
            trainer = None
            import gc

            gc.collect()
            torch.cuda.empty_cache()
            if i == len(candidates) - 1:
                raise
    dev_batches = [host[i].to(device) for i in range(accum)]

    def step(batches):
        m = None
        for b in batches:
            m = trainer.train_step({"input_ids": b})
        return m["loss"]

    # the fit probe above was one whole optimizer step: it counts as a warm-up step
    for _ in range(max(args.warmup - 1, 0)):
        step(dev_batches)
    sampler = ClockSampler(device_index=local_rank)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        _barrier_sync(dist, torch)
        e0.record()
        for _ in range(args.steps):
            loss = step(dev_batches)
        e1.record()
        _barrier_sync(dist, torch)
    dev_ms = _max_over_ranks(e0.elapsed_time(e1), dist, device)
    e2e = None
    if not args.no_e2e:
        n_e2e = max(1, min(args.steps, args.ref_e2e_steps))
        host_batches = [host[i] for i in range(accum)]
        _barrier_sync(dist, torch)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            lv = float(step(host_batches))
        _barrier_sync(dist, torch)
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dist, device)
        e2e = {"value": world * accum * micro * S * n_e2e / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": int(host.numel() * host.element_size()), "d2h_bytes_per_step": 4 * accum,
               "ms_per_step": e2e_s * 1000.0 / n_e2e, "steps": n_e2e}
    tokens_per_step = world * accum * micro * S
    res = {
        "metric": METRIC,
        "value": tokens_per_step * args.steps / (dev_ms / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (uniform token ids, seeded); random N(0,0.02) init",
        "impl": "reference",
        "config": {"model": MODEL_NAME, "global_batch": world * accum * micro, "seq_len": S, "micro_batch": micro,
                   "grad_accum": accum,
                   "parallelism": ("reference stock path, fp32, its vanilla attention: "
                                   + ("FSDP1 NO_SHARD" if world > 1 else "single GPU")),
                   "final_loss": float(loss)},
        "clocks": sampler.summary(),
        "e2e": e2e,
    }
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return res if rank == 0 else None


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        try:
            res = run_reference(args)
        except Exception as exc:  # report instead of crashing the driver
            res = {"impl": "reference", "unavailable": f"reference run failed: {type(exc).__name__}: {exc}"[:400]}
            if int(os.environ.get("RANK", 0)) != 0:
                res = None
    else:
        res = run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
