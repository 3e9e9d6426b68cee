"""Phase 1 with sharded data parallelism (``genesis/training/train_phase1_distributed.py:42-379``).

Launch: ``torchrun --nproc-per-node N -m genesis.training.train_phase1_distributed
--preset genesis-1b --data-dir packed/``.

:class:`DistributedBootstrapTrainer` reads ``LOCAL_RANK/WORLD_SIZE/RANK``,
initialises the process group (NCCL on GPUs, gloo on CPU), wraps the model
with the flat-shard engine (FULL_SHARD, bf16 compute, fp32 master) and uses
distributed Muon.  An explicitly passed ``fsdp_config`` is honoured on a
single GPU too (mixed precision through the same engine).

The reference ``main()`` fails while building its config
(``HLRTConfig(max_seq_len=...)``, ``train_phase1_distributed.py:288-291``);
this one builds the model from ``--preset`` (or the YAML given with
``--config``) and runs.
"""

from __future__ import annotations

import argparse
import logging
import math
import os
import time
from datetime import timedelta
from typing import Any, Dict, Optional

import torch
import torch.distributed as dist
from torch.utils.data import DataLoader
from torch.utils.data.distributed import DistributedSampler

from genesis.model.hlrt import HLRT
from genesis.training.train_phase1_bootstrap import ntp_objective
from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig
from olympus.data.tokenizer import TokenizerWrapper
from olympus.distributed.distributed_orchestrator import DistributedTrainingOrchestrator
from olympus.distributed.fsdp_wrapper import FSDPConfig
from olympus.optim.muon_adamw_hybrid import MuonAdamWHybrid
from olympus.optim.schedulers import WSDScheduler

logger = logging.getLogger(__name__)


def init_distributed(timeout_s: Optional[float] = None) -> tuple[int, int, int]:
    """Process group from the launcher's environment.  Collectives that do not
    finish within ``timeout_s`` (default ``LRB_PG_TIMEOUT_S`` or 600 s) are
    failed by NCCL's watchdog, and with asynchronous error handling on (the
    default set here unless the caller set ``TORCH_NCCL_ASYNC_ERROR_HANDLING``)
    the rank aborts its communicators and exits instead of hanging, so the
    launcher sees the failure."""
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    if timeout_s is None:
        timeout_s = float(os.environ.get("LRB_PG_TIMEOUT_S", 600.0))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
        if torch.cuda.is_available():
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s),
                                    device_id=torch.device("cuda", local_rank))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=timeout_s))
    return local_rank, world, rank


class DistributedBootstrapTrainer:
    def __init__(
        self,
        model: HLRT,
        optimizer_cls=MuonAdamWHybrid,
        optimizer_kwargs: Optional[dict] = None,
        scheduler_cls=WSDScheduler,
        scheduler_kwargs: Optional[dict] = None,
        tokenizer: Optional[TokenizerWrapper] = None,
        config: Optional[dict] = None,
        fsdp_config: Optional[FSDPConfig] = None,
    ) -> None:
        config = dict(config or {})
        self.local_rank, self.world_size, self.global_rank = init_distributed(config.get("dist_timeout_s"))
        self.is_distributed = self.world_size > 1
        if torch.cuda.is_available() and config.get("device", "cuda") != "cpu":
            self.device = torch.device(f"cuda:{self.local_rank}")
        else:
            self.device = torch.device("cpu")
        explicit = fsdp_config is not None
        if fsdp_config is None and self.is_distributed:
            fsdp_config = FSDPConfig(sharding_strategy="FULL_SHARD", mixed_precision="bf16",
                                     activation_checkpointing=config.get("activation_checkpointing", False))
        model = model.to(self.device)
        optimizer = optimizer_cls(model.parameters(), **(optimizer_kwargs or {}))
        scheduler = scheduler_cls(optimizer, **(scheduler_kwargs or {}))
        self.tokenizer = tokenizer or TokenizerWrapper(backend="tiktoken")
        self.sampler = None  # set by make_dataloader
        self._resume_position = None
        self.orchestrator = DistributedTrainingOrchestrator(
            fsdp_config=fsdp_config if (self.is_distributed or explicit) else None,
            local_rank=self.local_rank, world_size=self.world_size,
            gradient_accumulation_steps=config.get("gradient_accumulation_steps", 4),
            device=self.device, sync_metrics=config.get("sync_metrics", True),
        )
        self.orchestrator.add_model(ModelConfig(
            name="hlrt", model=model, optimizer=optimizer, scheduler=scheduler,
            max_grad_norm=config.get("max_grad_norm", 1.0), enabled_phases=["bootstrap"],
        ))
        self.orchestrator.add_objective(ObjectiveConfig(name="ntp", compute_fn=ntp_objective, weight=1.0,
                                                        enabled_phases=["bootstrap"]))
        self.orchestrator.set_phase("bootstrap")
        cfg = self.orchestrator._models["hlrt"]
        self.model, self.optimizer, self.scheduler = cfg.model, cfg.optimizer, cfg.scheduler
        self.config = config
        self._tokens_seen = 0

    @property
    def is_main_rank(self) -> bool:
        return self.global_rank == 0

    def train_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        t0 = time.time()
        losses = self.orchestrator.step(batch)
        total = losses.get("total", losses.get("ntp", 0.0))
        n = batch["input_ids"].numel()
        self._tokens_seen += n
        tps = n / max(time.time() - t0, 1e-6) * self.world_size
        if isinstance(total, torch.Tensor):
            ppl: Any = torch.where(total < 20, total.exp().clamp(max=1e6), torch.full_like(total, 1e6))
        else:
            ppl = min(math.exp(total), 1e6) if total < 20 else 1e6
        return {"loss": total, "perplexity": ppl, "lr": getattr(self.scheduler, "last_lr", 0.0), "tokens_per_sec": tps}

    def train_epoch(self, dataloader: DataLoader) -> Dict[str, float]:
        log_every = self.config.get("log_interval", 100)
        save_every = self.config.get("save_interval", 5000)
        ckpt_dir = self.config.get("checkpoint_dir", "checkpoints/phase1")
        tot, tps, steps = 0.0, 0.0, 0
        start = time.time()
        for batch in dataloader:
            m = self.train_step(batch)
            if self.sampler is not None and getattr(dataloader, "sampler", None) is self.sampler:
                self.sampler.advance(batch["input_ids"].shape[0])
            loss = float(m["loss"])
            tot += loss
            tps += m["tokens_per_sec"]
            steps += 1
            gs = self.orchestrator.global_step
            if self.is_main_rank and steps % log_every == 0:
                logger.info("Step %d | loss=%.4f | lr=%.2e | %.0f tok/s", gs, loss, m["lr"], m["tokens_per_sec"])
            if save_every > 0 and gs > 0 and gs % save_every == 0 and self.orchestrator._accumulation_step == 0:
                self.save_checkpoint(os.path.join(ckpt_dir, f"checkpoint_step{gs}.pt"))
            max_steps = self.config.get("max_steps")  # extension: stop inside the epoch at the step budget
            if max_steps is not None and gs >= max_steps and self.orchestrator._accumulation_step == 0:
                break
        avg = tot / max(steps, 1)
        if self.is_main_rank:
            logger.info("Epoch complete | avg_loss=%.4f | %d steps in %.1fs", avg, steps, time.time() - start)
        return {"epoch_loss": avg, "epoch_perplexity": min(math.exp(avg), 1e6) if avg < 20 else 1e6,
                "avg_tokens_per_sec": tps / max(steps, 1), "total_steps": steps}

    def save_checkpoint(self, path: str) -> None:
        if self.sampler is not None:  # extension: where in the epoch each rank stands
            states = [self.sampler.state_dict()]
            if self.is_distributed:
                states = [None] * self.world_size
                dist.all_gather_object(states, self.sampler.state_dict())
            self.orchestrator.extra_state["data_position"] = states
        self.orchestrator.save_checkpoint(path)

    def load_checkpoint(self, path: str) -> None:
        ckpt = self.orchestrator.load_checkpoint(path)
        self._resume_position = ckpt.get("data_position") if isinstance(ckpt, dict) else None
        if self.sampler is not None:
            self._apply_resume_position()

    def _apply_resume_position(self) -> None:
        pos = self._resume_position
        if pos and len(pos) == self.world_size:
            self.sampler.load_state_dict(pos[self.global_rank if self.is_distributed else 0])
        self._resume_position = None

    def make_dataloader(self, dataset, batch_size: int = 32, num_workers: int = 4) -> DataLoader:
        """Shuffled, split over the ranks, and resumable mid-epoch
        (:class:`olympus.data.resumable_sampler.ResumableDistributedSampler`)."""
        from olympus.data.resumable_sampler import ResumableDistributedSampler

        replicas = self.world_size if self.is_distributed else 1
        if len(dataset) // replicas < batch_size:
            raise ValueError(f"dataset of {len(dataset)} samples gives each of {replicas} rank(s) fewer than one "
                             f"batch of {batch_size} (drop_last=True): no training step would run")
        self.sampler = ResumableDistributedSampler(len(dataset), num_replicas=replicas,
                                                   rank=self.global_rank if self.is_distributed else 0, shuffle=True)
        if self._resume_position is not None:
            self._apply_resume_position()
        return DataLoader(dataset, batch_size=batch_size, sampler=self.sampler, num_workers=num_workers,
                          pin_memory=self.device.type == "cuda", drop_last=True)


def main(argv=None) -> None:
    from llm_research_b200.models.presets import build_hlrt_config

    ap = argparse.ArgumentParser(description="GENESIS phase-1 distributed training")
    ap.add_argument("--preset", default="genesis-1b")
    ap.add_argument("--config", default=None, help="YAML in the reference's nested schema (model, optimizer, "
                    "scheduler, training, hardware sections)")
    ap.add_argument("--set", dest="overrides", action="append", default=[], metavar="KEY.PATH=VALUE",
                    help="dotted override of the YAML, repeatable (e.g. --set model.tier1.layers=4)")
    ap.add_argument("--data-dir", default=None, help="packed data; synthetic tokens when omitted")
    ap.add_argument("--checkpoint-dir", default="checkpoints/phase1")
    ap.add_argument("--resume", default=None)
    # None: take the value from --config, else the default in brackets
    ap.add_argument("--max-steps", type=int, default=None, help="[50000]")
    ap.add_argument("--batch-size", type=int, default=None, help="[8]")
    ap.add_argument("--grad-accum", type=int, default=None, help="[4]")
    ap.add_argument("--lr", type=float, default=None, help="AdamW / base learning rate [3e-4]")
    ap.add_argument("--muon-lr", type=float, default=None, help="[0.02]")
    ap.add_argument("--warmup-steps", type=int, default=None, help="[2000]")
    ap.add_argument("--log-interval", type=int, default=None, help="[10]")
    ap.add_argument("--save-interval", type=int, default=None, help="[1000]")
    ap.add_argument("--seq-len", type=int, default=None, help="[4096]")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format=f"[rank {os.environ.get('RANK', 0)}] %(name)s | %(message)s")
    opt_kw: dict = {"lr_muon": 0.02, "lr_adamw": 3e-4, "weight_decay_adamw": 0.01, "ns_steps": 5}
    sched_kw: dict = {"min_lr": 2e-5}
    run = {"max_steps": 50000, "batch_size": 8, "gradient_accumulation_steps": 4, "log_interval": 10,
           "save_interval": 1000, "seq_len": 4096, "max_grad_norm": 1.0}
    if args.config:
        from olympus.utils.config import hlrt_config_from_yaml, load_config, parse_overrides, trainer_settings_from_yaml

        yaml_cfg = load_config(args.config, parse_overrides(args.overrides))
        cfg = hlrt_config_from_yaml(yaml_cfg)
        settings = trainer_settings_from_yaml(yaml_cfg)
        opt_kw.update(settings["optimizer_kwargs"])
        sched_kw.update(settings["scheduler_kwargs"])
        run.update({k: v for k, v in settings["trainer"].items() if k in run})
    else:
        if args.overrides:
            ap.error("--set needs --config")
        cfg = build_hlrt_config(args.preset)
    for flag, key in (("max_steps", "max_steps"), ("batch_size", "batch_size"), ("grad_accum", "gradient_accumulation_steps"),
                      ("log_interval", "log_interval"), ("save_interval", "save_interval"), ("seq_len", "seq_len")):
        if getattr(args, flag) is not None:
            run[key] = getattr(args, flag)
    if args.lr is not None:
        opt_kw["lr_adamw"] = sched_kw["base_lr"] = args.lr
    if args.muon_lr is not None:
        opt_kw["lr_muon"] = args.muon_lr
    if args.warmup_steps is not None:
        sched_kw["warmup_steps"] = args.warmup_steps
    sched_kw.setdefault("base_lr", opt_kw["lr_adamw"])
    sched_kw.setdefault("warmup_steps", 2000)
    sched_kw.setdefault("total_steps", run["max_steps"])
    sched_kw.setdefault("decay_start", int(sched_kw["total_steps"] * 0.9))
    torch.manual_seed(0)
    model = HLRT(cfg)
    trainer = DistributedBootstrapTrainer(
        model,
        optimizer_kwargs=opt_kw,
        scheduler_kwargs=sched_kw,
        tokenizer=TokenizerWrapper(backend="char", vocab_size=cfg.vocab_size),
        config={"gradient_accumulation_steps": run["gradient_accumulation_steps"], "max_grad_norm": run["max_grad_norm"],
                "log_interval": run["log_interval"], "save_interval": run["save_interval"],
                "checkpoint_dir": args.checkpoint_dir, "max_steps": run["max_steps"]},
    )
    if args.resume:
        trainer.load_checkpoint(args.resume)
    if args.data_dir:
        from olympus.data.packed_dataset import PackedDataset

        ds = PackedDataset(args.data_dir, split="train")
    else:
        from olympus.data.packed_dataset import SyntheticTokenDataset

        ds = SyntheticTokenDataset(max(run["batch_size"] * trainer.world_size * 64, 64), run["seq_len"], cfg.vocab_size)
    loader = trainer.make_dataloader(ds, batch_size=run["batch_size"], num_workers=2)
    epoch = trainer.sampler.epoch  # the resumed epoch, 0 on a fresh start
    empty_epochs = 0
    while trainer.orchestrator.global_step < run["max_steps"]:
        if hasattr(loader.sampler, "set_epoch"):
            loader.sampler.set_epoch(epoch)
        trainer.orchestrator.set_epoch(epoch)
        ran = trainer.train_epoch(loader)["total_steps"]
        epoch += 1
        # A resumed epoch may already be used up; a second empty epoch in a row
        # means the loader yields nothing and the loop would never end.
        empty_epochs = empty_epochs + 1 if ran == 0 else 0
        if empty_epochs >= 2:
            raise RuntimeError("two epochs in a row yielded no batch; the dataset is too small for the batch size")
    trainer.save_checkpoint(os.path.join(args.checkpoint_dir, "checkpoint_final.pt"))
    if trainer.is_distributed:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
