"""Fused compute + collective paths on N GPUs of one node, against the NCCL baseline.

``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m llm_research_b200.comm_bench``

For every case the time is measured with CUDA events on each rank (warm-up,
synchronise + barrier on both sides) and the MAX over ranks is reported; one
JSON line per case on rank 0 with the achieved fraction of its roofline:
``max(FLOPs / measured bf16 GEMM peak, bytes each GPU must send over NVLink /
770 GB/s per direction)``.

Cases (M = tokens over all ranks, sequence-sharded; N x K weights):
  ag_gemm      fused all-gather(rows) -> GEMM    vs  NCCL all_gather + cuBLAS
  gemm_rs      fused GEMM -> reduce-scatter(rows) vs  cuBLAS + NCCL reduce_scatter
  tp_rows_*    the P2P row all-gather and reduce-scatter (+ residual) that the NVFP4 TP layers
               run around their block-scaled GEMMs  vs  NCCL
  fsdp_rs      P2P reduce-scatter (bf16 wire, fp32 accumulate, fused norm) vs NCCL (fp32)
  ep_dispatch  MoE dispatch (P2P stores into the owners' expert slots) vs NCCL all_to_all
  ep_combine   MoE combine (P2P loads fused with the top-k weighted sum) vs NCCL all_to_all + gather
               (``--ep-tokens`` per rank x d 4096, top-2 of 16 experts, random-normal router logits)
  nvls_rs      FSDP reduce-scatter through NVSwitch multicast (bf16 staging, multimem.ld_reduce
               summing in the switch, fused scale/norm) vs NCCL (fp32)
  nvls_ag      once-per-step parameter broadcast (fp32 master shard -> bf16 multimem.st into every
               rank's gathered buffer) vs NCCL all_gather of the bf16 shards
  nvls_ar      in-place fp32 all-reduce (multimem.ld_reduce of one slice per rank, multimem.st of
               the sum) vs NCCL all_reduce, ``--ar-elements`` per rank
  diloco_outer DiLoCo outer step over all ranks as replicas (fused pseudo-gradient exchange +
               Nesterov on symmetric memory) vs the all-reduce path, ``--diloco-elements`` fp32
               per rank
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _peak_tflops() -> float:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def _time(fn, warmup: int, iters: int, dev) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="+", default=[8192, 32768])
    ap.add_argument("--nk", type=int, nargs="+", default=[4096, 8192])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--ep-tokens", type=int, nargs="*", default=[1024, 8192, 65536])
    ap.add_argument("--nvls", type=int, default=1, help="run the NVSwitch multicast cases (0: skip)")
    ap.add_argument("--ar-elements", type=int, nargs="*", default=[16 * 1024 * 1024, 128 * 1024 * 1024])
    ap.add_argument("--diloco-elements", type=int, default=0,
                    help="per-rank fp32 elements of the DiLoCo outer-step case (0: skip)")
    args = ap.parse_args(argv)
    import datetime

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from llm_research_b200.parallel.tp import TPComm

    peak = _peak_tflops()
    maxT, maxW = max(args.tokens), max(args.nk)
    comm = TPComm(None, max_tokens=maxT, max_width=maxW, device=dev)

    def report(case, T, N, K, ms, base_ms, flops, nvbytes):
        if rank != 0:
            return
        roof_ms = max(flops / (peak * 1e12), nvbytes / (NVLINK_GBS * 1e9)) * 1e3
        print(json.dumps({"case": case, "gpus": world, "M": T, "N": N, "K": K, "ms": round(ms, 4),
                          "nccl_ms": round(base_ms, 4), "speedup_vs_nccl": round(base_ms / ms, 3),
                          "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3)}), flush=True)

    for T in args.tokens:
        for NK in args.nk:
            N = K = NK
            Tl = T // world
            x_shard = torch.randn(Tl, K, device=dev, dtype=torch.bfloat16)
            w = torch.randn(N // world, K, device=dev, dtype=torch.bfloat16) * 0.02  # column shard
            full = torch.empty(T, K, device=dev, dtype=torch.bfloat16)

            def nccl_ag():
                dist.all_gather_into_tensor(full, x_shard)
                return full @ w.t()

            flops = 2.0 * T * (N // world) * K
            ag_bytes = (world - 1) * Tl * K * 2
            ms = _time(lambda: comm.ag_gemm(x_shard, w), args.warmup, args.iters, dev)
            base = _time(nccl_ag, args.warmup, args.iters, dev)
            report("ag_gemm", T, N // world, K, ms, base, flops, ag_bytes)

            xk = torch.randn(T, K // world, device=dev, dtype=torch.bfloat16)  # row-parallel input
            w2 = torch.randn(N, K // world, device=dev, dtype=torch.bfloat16) * 0.02
            out = torch.empty(Tl, N, device=dev, dtype=torch.bfloat16)

            def nccl_rs():
                y = xk @ w2.t()
                dist.reduce_scatter_tensor(out, y)
                return out

            flops = 2.0 * T * N * (K // world)
            rs_bytes = (world - 1) * Tl * N * 2
            ms = _time(lambda: comm.gemm_rs(xk, w2), args.warmup, args.iters, dev)
            base = _time(nccl_rs, args.warmup, args.iters, dev)
            report("gemm_rs", T, N, K // world, ms, base, flops, rs_bytes)

            # the row collectives the NVFP4 layers run around their block-scaled GEMMs
            y = torch.randn(T, N, device=dev, dtype=torch.bfloat16)
            res = torch.randn(Tl, N, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: comm.all_gather(x_shard), args.warmup, args.iters, dev)
            base = _time(lambda: dist.all_gather_into_tensor(full, x_shard), args.warmup, args.iters, dev)
            report("tp_rows_all_gather", T, 0, K, ms, base, 0.0, ag_bytes)
            ms = _time(lambda: comm.reduce_scatter(y, res), args.warmup, args.iters, dev)

            def nccl_rows_rs():
                dist.reduce_scatter_tensor(out, y)
                return out + res

            base = _time(nccl_rows_rs, args.warmup, args.iters, dev)
            report("tp_rows_reduce_scatter_residual", T, N, 0, ms, base, 0.0, rs_bytes)
            del x_shard, w, full, xk, w2, out, y, res
    comm.heap.check()
    comm.close()

    # FSDP gradient reduce-scatter of a 7B-sized unit (fp32 accumulators)
    from llm_research_b200._ext import native
    from llm_research_b200.parallel.symm import SymmetricHeap

    C = native()
    n = 8 * 1024 * 1024 * world  # elements per unit
    shard = n // world
    heap = SymmetricHeap(world * shard * 2 + 8192, device=dev)
    recv_off, ready_off, consumed_off = heap.alloc(world * shard * 2), heap.alloc(4 * world), heap.alloc(4)
    recv = heap.view(recv_off, (world * shard,), torch.bfloat16)
    ready, consumed = heap.view(ready_off, (world,), torch.int32), heap.view(consumed_off, (1,), torch.int32)
    counters = torch.zeros(4, dtype=torch.int32, device=dev)
    g = torch.randn(n, device=dev)
    dst = torch.empty(shard, device=dev)
    sumsq = torch.zeros((), device=dev)
    state = {"e": 0}

    def p2p():
        state["e"] += 1
        C.p2p_rs_push(g, heap.bases, recv_off, ready_off, consumed_off, rank, world, shard, state["e"], counters[0:1],
                      heap.err)
        C.p2p_rs_reduce(recv, dst, world, 1.0 / world, False, ready, consumed, state["e"], sumsq, counters[1:2],
                        heap.err)

    def nccl():
        dist.reduce_scatter_tensor(dst, g, op=dist.ReduceOp.AVG)

    ms = _time(p2p, args.warmup, args.iters, dev)
    base = _time(nccl, args.warmup, args.iters, dev)
    if rank == 0:
        roof = (world - 1) * shard * 2 / (NVLINK_GBS * 1e9) * 1e3
        print(json.dumps({"case": "fsdp_rs", "gpus": world, "elements": n, "ms": round(ms, 4), "nccl_fp32_ms": round(base, 4),
                          "speedup_vs_nccl": round(base / ms, 3), "roofline_ms": round(roof, 4),
                          "frac_of_roofline": round(roof / ms, 3)}), flush=True)
    heap.check()
    heap.close()
    if args.nvls:
        _nvls_cases(args, rank, world, dev, n)
    if args.ep_tokens:
        _ep_cases(args, rank, world, dev)
    if args.diloco_elements:
        _diloco_case(args, rank, world, dev)
    dist.barrier()
    dist.destroy_process_group()


def _nvls_cases(args, rank: int, world: int, dev, n: int) -> None:
    """The multicast (NVLS) collectives against NCCL; skipped without multicast."""
    from llm_research_b200._ext import native
    from llm_research_b200.parallel.nvls import MulticastHeap, NVLSAllReduce, NVLSUnavailable

    C = native()
    shard = n // world
    try:
        heap = MulticastHeap(2 * n * 2 + 4 * sum(args.ar_elements or [0]) + (1 << 22), device=dev)
    except NVLSUnavailable as e:
        if rank == 0:
            print(json.dumps({"case": "nvls", "gpus": world, "skipped": str(e)}), flush=True)
        return
    stage_off, ag_off, flag_off = heap.alloc(n * 2), heap.alloc(n * 2), heap.alloc(16 * world)
    stage = heap.view(stage_off, (n,), torch.bfloat16)
    flags = heap.view(flag_off, (4 * world,), torch.int32)
    ready, consumed, agfree, agready = (flags[i * world:(i + 1) * world] for i in range(4))
    counters = torch.zeros(4, dtype=torch.int32, device=dev)
    g = torch.randn(n, device=dev)
    dst = torch.empty(shard, device=dev)
    sumsq = torch.zeros((), device=dev)
    master = torch.randn(shard, device=dev)
    full = torch.empty(n, dtype=torch.bfloat16, device=dev)
    master_bf = master.to(torch.bfloat16)
    st = {"rs": 0, "ag": 0}

    def rs():
        st["rs"] += 1
        C.nvls_rs_stage(g, stage, consumed, heap.bases, flag_off, rank, world, st["rs"], counters[0:1], heap.err)
        C.nvls_rs_reduce(heap.mc(stage_off), dst, 1.0 / world, False, ready, heap.bases, flag_off + 4 * world, rank,
                         world, st["rs"], sumsq, counters[1:2], heap.err)

    def ag():
        st["ag"] += 1
        C.nvls_ag_publish(master, heap.mc(ag_off), agfree, heap.bases, flag_off + 8 * world, flag_off + 12 * world,
                          rank, world, st["ag"], counters[2:3], heap.err)
        C.nvls_wait(agready, world, st["ag"], heap.err)

    ms_rs = _time(rs, args.warmup, args.iters, dev)
    base_rs = _time(lambda: dist.reduce_scatter_tensor(dst, g, op=dist.ReduceOp.AVG), args.warmup, args.iters, dev)
    ms_ag = _time(ag, args.warmup, args.iters, dev)
    base_ag = _time(lambda: dist.all_gather_into_tensor(full, master_bf), args.warmup, args.iters, dev)
    if rank == 0:
        roof = (world - 1) * shard * 2 / (NVLINK_GBS * 1e9) * 1e3  # bf16 bytes that must reach / leave each GPU
        for case, ms, base, what in (("nvls_rs", ms_rs, base_rs, "nccl_fp32_ms"),
                                     ("nvls_ag", ms_ag, base_ag, "nccl_bf16_ms")):
            print(json.dumps({"case": case, "gpus": world, "elements": n, "ms": round(ms, 4), what: round(base, 4),
                              "speedup_vs_nccl": round(base / ms, 3), "roofline_ms": round(roof, 4),
                              "frac_of_roofline": round(roof / ms, 3)}), flush=True)
    for m in args.ar_elements:
        ar = NVLSAllReduce(m, heap=heap)
        ar.tensor().normal_()
        x = torch.randn(m, device=dev)
        ms = _time(ar.run, args.warmup, args.iters, dev)
        base = _time(lambda: dist.all_reduce(x), args.warmup, args.iters, dev)
        if rank == 0:
            # each GPU's data leaves once and the sum arrives once (bytes per direction)
            roof = m * 4 * (world - 1) / world / (NVLINK_GBS * 1e9) * 1e3
            print(json.dumps({"case": "nvls_ar", "gpus": world, "elements": m, "ms": round(ms, 4),
                              "nccl_ms": round(base, 4), "speedup_vs_nccl": round(base / ms, 3),
                              "busbw_gbs": round(2 * (world - 1) / world * m * 4 / ms / 1e6, 1),
                              "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / ms, 3)}), flush=True)
    heap.check()
    heap.close()


def _ep_cases(args, rank: int, world: int, dev) -> None:
    """MoE dispatch / combine at T tokens per rank, d 4096, top-2 of 16 experts."""
    import math

    from llm_research_b200 import ops
    from llm_research_b200.parallel.expert_parallel import EPComm, _combine_collective, _dispatch_collective, make_route

    E, K, D = 16, 2, 4096
    if E % world:
        return
    epl = E // world
    comm = EPComm(None, max_tokens=max(args.ep_tokens), top_k=K, d=D, experts_per_rank=epl, capacity_factor=1.25,
                  device=dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    for T in args.ep_tokens:
        x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, device=dev, generator=g)
        w, idx, _ = ops.softmax_topk(logits, K)
        cap = math.ceil(1.25 * T * K / E)
        route = make_route(idx, epl, E, cap)
        xe = torch.randn(epl, world * cap, D, device=dev, generator=g).to(torch.bfloat16)
        wf = w.reshape(-1).float().contiguous()

        def fused_dispatch():
            comm.push(x, None, False, route, cap, K)
            return comm.take(cap)

        def fused_combine():
            comm.put(xe, cap)
            return comm.pull(T, wf, False, route, cap, K)

        ms_d = _time(fused_dispatch, args.warmup, args.iters, dev)
        base_d = _time(lambda: _dispatch_collective(x, route, cap, world, epl, None), args.warmup, args.iters, dev)
        ms_c = _time(fused_combine, args.warmup, args.iters, dev)
        base_c = _time(lambda: _combine_collective(xe, w, route, cap, world, epl, None), args.warmup, args.iters, dev)
        if rank == 0:
            # rows that leave this GPU: the (world-1)/world share of its T*K assignments
            nv = T * K * (world - 1) / world * D * 2
            roof = nv / (NVLINK_GBS * 1e9) * 1e3
            for case, ms, base in (("ep_dispatch", ms_d, base_d), ("ep_combine", ms_c, base_c)):
                print(json.dumps({"case": case, "gpus": world, "tokens_per_rank": T, "d": D, "experts": E,
                                  "top_k": K, "ms": round(ms, 4), "nccl_ms": round(base, 4),
                                  "speedup_vs_nccl": round(base / ms, 3), "roofline_ms": round(roof, 4),
                                  "frac_of_roofline": round(roof / ms, 3)}), flush=True)
    comm.close()



def _diloco_case(args, rank: int, world: int, dev) -> None:
    """One outer step of DiLoCo with every rank a replica: P2P (push pseudo-gradient
    slices to their owners, fused average + Nesterov, pull the new anchor) against
    the collective path (all-reduce of the pseudo-gradient, local Nesterov)."""
    from llm_research_b200.parallel.diloco import DiLoCo, DiLoCoConfig

    n = args.diloco_elements
    shard = torch.randn(n, device=dev)
    times = {}
    for comm in ("p2p", "nvls", "collective"):
        dl = DiLoCo([shard], dist.group.WORLD, list(range(world)),
                    DiLoCoConfig(comm=comm, fault_tolerance=False), tag=f"bench-{comm}")
        if dl.comm == comm:
            times[comm] = _time(dl.outer_step, args.warmup, args.iters, dev)
        dl.close()
    if rank == 0:
        # each rank sends (world-1)/world of its fp32 pseudo-gradient and receives the same of the anchor
        nv = n * 4 * (world - 1) / world
        roof = nv / (NVLINK_GBS * 1e9) * 1e3
        print(json.dumps({"case": "diloco_outer", "gpus": world, "elements_per_rank": n,
                          "ms": round(times["p2p"], 4), "collective_ms": round(times["collective"], 4),
                          "speedup_vs_nccl": round(times["collective"] / times["p2p"], 3),
                          "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / times["p2p"], 3)}),
              flush=True)
        if "nvls" in times:
            print(json.dumps({"case": "diloco_outer_nvls", "gpus": world, "elements_per_rank": n,
                              "ms": round(times["nvls"], 4), "collective_ms": round(times["collective"], 4),
                              "speedup_vs_nccl": round(times["collective"] / times["nvls"], 3),
                              "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / times["nvls"], 3)}),
                  flush=True)


if __name__ == "__main__":
    main()
