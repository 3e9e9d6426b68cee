"""Sharded, asynchronous checkpoints of the flat-shard engine, and their
consolidation into the single-file layout of the reference
(``olympus/core/training_orchestrator.py:225-278``: ``models[name]`` holds the
full tensors by parameter name).

``save_sharded(engine, optimizer, dir, header)``: every rank copies its fp32
master shards, its optimizer-state shards and its rank-local parameters to
host memory and writes ``rank{r:05d}.pt`` from a background thread (the
training loop continues once the device-to-host copies are done); rank 0
also writes ``layout.pt`` (parameter -> unit / offset / shape, world size)
and the caller's ``header`` (step, phase, scheduler state, buffers, ...).
``wait()`` joins the writer threads.

``load_sharded(engine, optimizer, dir)``: same world size -> each rank reads
its own file; otherwise the shards are consolidated first and loaded as full
tensors.

``consolidate(dir)``: a full checkpoint dict (``models``, ``optimizer_state``
by parameter name, plus the header) built on the host from the shard files;
``consolidate_checkpoint(dir)`` does the same for a whole orchestrator
checkpoint; ``python -m llm_research_b200.parallel.checkpoint DIR OUT.pt``
writes it.
"""

from __future__ import annotations

import os
import sys
import threading
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist

_WRITERS: List[threading.Thread] = []


def _host(t: torch.Tensor) -> torch.Tensor:
    if t.device.type == "cpu":
        return t.detach().clone()
    out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    out.copy_(t.detach(), non_blocking=True)
    return out


def _shard_state(engine, optimizer) -> Dict[str, Any]:
    units = [{"index": u.index, "total": u.total, "shard": u.shard, "master": _host(u.master)} for u in engine.units]
    opt: Dict[str, Any] = {}
    for key in ("momentum", "exp_avg", "exp_avg_sq"):
        bufs = getattr(optimizer, key, None)
        if isinstance(bufs, dict):
            opt[key] = {ui: _host(b) for ui, b in bufs.items()}
    if hasattr(optimizer, "steps"):
        opt["steps"] = dict(optimizer.steps)
    local = {name: _host(p) for name, p in engine.local_params}
    local_mom = {name: _host(b) for name, b in getattr(optimizer, "local_momentum", {}).items()}
    return {"rank": engine.rank, "world": engine.world, "units": units, "optimizer": opt, "local": local,
            "local_momentum": local_mom}


def _layout(engine) -> Dict[str, Any]:
    return {"world": engine.world,
            "params": [{"name": i.name, "unit": i.unit, "offset": i.offset, "shape": tuple(i.shape),
                        "numel": i.numel, "index": i.index} for i in engine.params],
            "units": [{"index": u.index, "total": u.total, "shard": u.shard} for u in engine.units]}


def save_sharded(engine, optimizer, directory: str, header: Optional[Dict[str, Any]] = None,
                 asynchronous: bool = True, rank_extra: Optional[Dict[str, Any]] = None) -> None:
    """``header``: rank 0's metadata; ``rank_extra``: this rank's own entries (its RNG
    states, say), returned by :func:`load_sharded` when the world size is unchanged."""
    os.makedirs(directory, exist_ok=True)
    state = _shard_state(engine, optimizer)
    state["extra"] = dict(rank_extra or {})
    if engine.device.type == "cuda":
        torch.cuda.synchronize(engine.device)  # host copies complete before the writer reads them
    path = os.path.join(directory, f"rank{engine.rank:05d}.pt")
    jobs = [(state, path)]
    if engine.rank == 0:
        jobs.append(({"layout": _layout(engine), "header": header or {}}, os.path.join(directory, "layout.pt")))

    def write() -> None:
        for obj, p in jobs:
            tmp = p + ".tmp"
            torch.save(obj, tmp)
            os.replace(tmp, p)

    if asynchronous:
        t = threading.Thread(target=write, name="lrb-ckpt-writer", daemon=False)
        t.start()
        _WRITERS.append(t)
    else:
        write()


def wait() -> None:
    while _WRITERS:
        _WRITERS.pop().join()


def _load_rank(directory: str, rank: int) -> Dict[str, Any]:
    return torch.load(os.path.join(directory, f"rank{rank:05d}.pt"), map_location="cpu", weights_only=False)


@torch.no_grad()
def load_sharded(engine, optimizer, directory: str) -> Dict[str, Any]:
    meta = torch.load(os.path.join(directory, "layout.pt"), map_location="cpu", weights_only=False)
    out = dict(meta["header"])
    if meta["layout"]["world"] == engine.world:
        st = _load_rank(directory, engine.rank)
        out.update(st.get("extra", {}))
        for u, s in zip(engine.units, st["units"]):
            u.master.copy_(s["master"].to(u.master.device))
        for key, bufs in st["optimizer"].items():
            if key == "steps":
                optimizer.steps.clear()
                optimizer.steps.update(bufs)
                continue
            dst = getattr(optimizer, key, None)
            if isinstance(dst, dict):
                for ui, b in bufs.items():
                    if ui in dst:
                        dst[ui].copy_(b.to(dst[ui].device))
    else:
        full = consolidate(directory)
        engine.load_full_state_dict(full["models"]["model"])
        st = _load_rank(directory, engine.rank % meta["layout"]["world"])
    local = dict(engine.local_params)
    for name, t in st["local"].items():
        if name in local:
            local[name].copy_(t.to(local[name].device))
    if hasattr(optimizer, "local_momentum"):
        for name, t in st.get("local_momentum", {}).items():
            optimizer.local_momentum[name] = t.to(engine.device)
    engine.refresh()
    if dist.is_available() and dist.is_initialized() and engine.world > 1:
        dist.barrier(group=engine.pg)
    return out


def consolidate(directory: str, model_name: str = "model") -> Dict[str, Any]:
    meta = torch.load(os.path.join(directory, "layout.pt"), map_location="cpu", weights_only=False)
    lay = meta["layout"]
    W = lay["world"]
    ranks = [_load_rank(directory, r) for r in range(W)]
    full_units = {}
    opt_full: Dict[str, Dict[int, torch.Tensor]] = {}
    for u in lay["units"]:
        ui = u["index"]
        full_units[ui] = torch.cat([rk["units"][ui]["master"] for rk in ranks]) if W > 1 else ranks[0]["units"][ui]["master"]
        for key in ("momentum", "exp_avg", "exp_avg_sq"):
            pieces = [rk["optimizer"].get(key, {}).get(ui) for rk in ranks]
            if all(p is not None for p in pieces):
                opt_full.setdefault(key, {})[ui] = torch.cat(pieces) if W > 1 else pieces[0]
    model: Dict[str, torch.Tensor] = {}
    opt_state: Dict[str, Dict[str, torch.Tensor]] = {}
    for p in lay["params"]:
        sl = slice(p["offset"], p["offset"] + p["numel"])
        model[p["name"]] = full_units[p["unit"]][sl].view(p["shape"]).clone()
        for key, per_unit in opt_full.items():
            if p["unit"] in per_unit:
                opt_state.setdefault(p["name"], {})[key] = per_unit[p["unit"]][sl].view(p["shape"]).clone()
    for rk in ranks:  # rank-local parameters (expert parallelism) keep their rank in the name
        for name, t in rk["local"].items():
            model[f"{name}@rank{rk['rank']}"] = t
    header = dict(meta["header"])
    ckpt = {k: v for k, v in header.items() if k not in ("models",)}
    ckpt["models"] = {model_name: {**header.get("buffers", {}), **model}}
    ckpt["optimizer_state"] = {model_name: opt_state}
    ckpt["world_size"] = W
    return ckpt


def consolidate_checkpoint(directory: str) -> Dict[str, Any]:
    """A directory written by ``DistributedTrainingOrchestrator.save_sharded_checkpoint`` as one
    checkpoint dict in the reference's layout (``global_step``, ``epoch``, ``phase``, ``prev_loss``,
    ``memory_bus``, ``models``/``optimizers``/``schedulers`` by model name). Engine-wrapped models
    contribute full tensors by parameter name; their optimizer state goes under ``optimizer_state``
    (per parameter) because the sharded optimizer has no single-process ``state_dict``."""
    head_path = os.path.join(directory, "header.pt")
    if not os.path.exists(head_path):  # a bare engine directory
        return consolidate(directory)
    head = torch.load(head_path, map_location="cpu", weights_only=False)
    ckpt = {k: v for k, v in head.items() if k != "sharded"}
    ckpt.setdefault("optimizer_state", {})
    for name in head.get("sharded", []):
        sub = consolidate(os.path.join(directory, name), model_name=name)
        ckpt["models"][name] = sub["models"][name]
        ckpt["optimizer_state"][name] = sub["optimizer_state"][name]
    return ckpt


def main(argv=None) -> None:
    args = sys.argv[1:] if argv is None else argv
    if len(args) != 2:
        print("usage: python -m llm_research_b200.parallel.checkpoint SHARD_DIR OUT.pt")
        raise SystemExit(2)
    torch.save(consolidate_checkpoint(args[0]), args[1])


if __name__ == "__main__":
    main()
