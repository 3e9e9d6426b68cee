"""Per-kernel microbenchmarks on one GPU.

``python -m llm_research_b200.kernel_bench [names...] [--iters N] [--warmup W]``
times each kernel with CUDA events on the launching stream (after warm-up,
synchronised on both sides), writes a 256 MiB buffer between timed
iterations so that every iteration starts with a cold L2, and prints one JSON
line per case with the achieved FLOP/s or bytes/s and its fraction of the
measured peaks in ``MEASURED_PEAKS.json`` at the repository root (the copy
bandwidth and the cuBLAS bf16 GEMM burst rate).

The same command with ``--iters 1 --warmup 1`` is the small case used for
Nsight Compute captures of one kernel.

Cases (shapes are the GENESIS-1B / 7B working shapes):
  attn_fwd, attn_bwd     causal flash attention, B=4, S=4096, H=16, hd=128 (tcgen05)
  attn_fwd_gqa           B=2, S=4096, H=32, Hkv=8, hd=128
  gemm                   tcgen05 bf16 GEMM 8192x8192x8192 (TN)
  gemm_cublas            the same shape through torch.matmul (library reference)
  gemm_pair              CTA-pair tcgen05 GEMM (cta_group::2) 8192x8192x8192
  lin_<name>_<kind>[_cublas]  fwd / dgrad / wgrad GEMM of a GENESIS-1B linear at
                         32768 tokens (qkv, o, upgate, down, head), pair kernel or cuBLAS
  gemm_nvfp4             tcgen05 block-scaled NVFP4 GEMM 8192x8192x8192 (nominal FP4 dense peak 4.5 PFLOP/s)
  rmsnorm_fwd/bwd        32768 x 2048 bf16
  swiglu_fwd             32768 x (2 x 5632) bf16
  ns                     Newton-Schulz, 5 iterations, batch 8 of 2048 x 5632
  ce                     cross-entropy fwd+bwd, 32768 x 32000 bf16 logits
"""

from __future__ import annotations

import argparse
import json
import math
import os
from typing import Callable, Dict, Tuple

import torch

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peaks() -> Dict[str, float]:
    path = os.path.join(_REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class _Timer:
    def __init__(self, warmup: int, iters: int) -> None:
        self.warmup, self.iters = warmup, iters
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def __call__(self, fn: Callable[[], None]) -> float:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(self.iters):
            self.flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        return total / self.iters


def _attn_case(B: int, S: int, H: int, Hkv: int, bwd: bool) -> Tuple[Callable[[], None], float, float]:
    from llm_research_b200._ext import native

    C = native()
    q = torch.randn(B, S, H, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    flops = 4.0 * B * H * S * S * 128 / 2  # causal: half of QK^T and PV
    if not bwd:
        return (lambda: C.attn_fwd_sm100(q, k, v, True, scale)), flops, 0.0
    o, lse = C.attn_fwd_sm100(q, k, v, True, scale)
    do = torch.randn_like(o)
    return (lambda: C.attn_bwd(do, q, k, v, o, lse, True, scale, True)), 2.5 * flops, 0.0


def _cases() -> Dict[str, Callable[[], Tuple[Callable[[], None], float, float]]]:
    from llm_research_b200._ext import native

    C = native()

    def gemm(lib: bool):
        n = 8192
        a = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        if lib:
            return (lambda: torch.matmul(a, b.t())), 2.0 * n ** 3, 0.0
        return (lambda: C.gemm_tn(a, b, torch.bfloat16, 1.0)), 2.0 * n ** 3, 0.0

    def gemm_pair():
        n = 8192
        a = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(n, n, device="cuda", dtype=torch.bfloat16)
        return (lambda: C.gemm_pair(a, b, False, False, c, False, 1.0)), 2.0 * n ** 3, 0.0

    def gemm_fp4():
        from llm_research_b200.ops.quant import NVFP4Tensor, matmul_nvfp4

        n = 8192
        a = NVFP4Tensor.quantize(torch.randn(n, n, device="cuda", dtype=torch.bfloat16))
        b = NVFP4Tensor.quantize(torch.randn(n, n, device="cuda", dtype=torch.bfloat16))
        return (lambda: matmul_nvfp4(a, b)), 2.0 * n ** 3, 0.0

    def quant_dual():
        from llm_research_b200.ops.quant import nvfp4_quantize_dual

        x = torch.randn(8192, 4096, device="cuda", dtype=torch.bfloat16)
        # one read of x, both FP4 copies with their scales written
        return (lambda: nvfp4_quantize_dual(x)), 0.0, x.numel() * (2 + 2 * (0.5 + 1 / 16))

    def linear_train(precision: str):
        from llm_research_b200.ops.linear import linear_precision, project

        T, K, N = 8192, 4096, 11008
        x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02).requires_grad_()
        dy = torch.randn(T, N, device="cuda", dtype=torch.bfloat16)

        def run():
            with linear_precision(precision):
                x.grad = w.grad = None
                project(x, w).backward(dy)

        return run, 6.0 * T * K * N, 0.0

    def memory_read():
        import torch.nn.functional as F

        from llm_research_b200.ops.memory import bank_read

        T, N, D = 8192, 65536, 4096  # one micro-batch of 2 x 4096 tokens against the 7B bank
        keys = F.normalize(torch.randn(N, D, device="cuda"), dim=-1).to(torch.bfloat16)
        values = torch.randn(N, D, device="cuda", dtype=torch.bfloat16)
        q = torch.randn(T, D, device="cuda", dtype=torch.bfloat16)
        return (lambda: bank_read(q, keys, values, 32)), 2.0 * T * N * D, 0.0

    def rms(bwd: bool):
        rows, d = 32768, 2048
        x = torch.randn(rows, d, device="cuda", dtype=torch.bfloat16)
        w = torch.ones(d, device="cuda", dtype=torch.bfloat16)
        y, rstd, _ = C.rmsnorm_fwd(x, w, 1e-6, None, torch.bfloat16)
        if not bwd:
            return (lambda: C.rmsnorm_fwd(x, w, 1e-6, None, torch.bfloat16)), 0.0, 2.0 * x.numel() * 2
        dy = torch.randn_like(y)
        return (lambda: C.rmsnorm_bwd(dy, x, w, rstd, None)), 0.0, 3.0 * x.numel() * 2

    def swiglu():
        from llm_research_b200 import ops

        gu = torch.randn(32768, 2 * 5632, device="cuda", dtype=torch.bfloat16)
        return (lambda: ops.swiglu(gu)), 0.0, gu.numel() * 2 * 1.5

    def ns_shape(m, n, batch):
        from llm_research_b200 import ops

        g = torch.randn(batch, m, n, device="cuda", dtype=torch.bfloat16)
        s, l = min(m, n), max(m, n)
        flops = batch * 5 * (2 * s * s * l + 2 * s * s * s + 2 * s * s * l)
        return (lambda: ops.newton_schulz(g, steps=5)), float(flops), 0.0

    def ns():
        from llm_research_b200 import ops

        g = torch.randn(8, 2048, 5632, device="cuda", dtype=torch.bfloat16)
        m, n = 2048, 5632
        flops = 8 * 5 * (2 * m * m * n + 2 * m * m * m + 2 * m * m * n)
        return (lambda: ops.newton_schulz(g, steps=5)), float(flops), 0.0

    def ce():
        from llm_research_b200 import ops

        logits = torch.randn(32768, 32000, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        tgt = torch.randint(0, 32000, (32768,), device="cuda")

        def run():
            logits.grad = None
            ops.cross_entropy(logits, tgt).backward()

        return run, 0.0, logits.numel() * 2 * 3.0

    cases = {
        "attn_fwd": lambda: _attn_case(4, 4096, 16, 16, False),
        "attn_bwd": lambda: _attn_case(4, 4096, 16, 16, True),
        "attn_fwd_gqa": lambda: _attn_case(2, 4096, 32, 8, False),
        "gemm": lambda: gemm(False),
        "gemm_cublas": lambda: gemm(True),
        "gemm_nvfp4": gemm_fp4,
        "nvfp4_quant_dual": quant_dual,
        "memory_read": memory_read,
        "linear_fwd_bwd_bf16": lambda: linear_train("bf16"),
        "linear_fwd_bwd_nvfp4": lambda: linear_train("nvfp4"),
        "rmsnorm_fwd": lambda: rms(False),
        "rmsnorm_bwd": lambda: rms(True),
        "swiglu_fwd": swiglu,
        "ns": ns,
        "ns_4096x4096": lambda: ns_shape(4096, 4096, 8),
        "ns_4096x11008": lambda: ns_shape(4096, 11008, 8),
        "ce": ce,
        "gemm_pair": gemm_pair,
    }
    cases["lin_upgate_swiglu"] = _swiglu_up_case
    cases["lin_qkv_rope"] = _qkv_rope_case
    for name, (N, K) in LINEAR_SHAPES.items():
        for kind in ("fwd", "dgrad", "wgrad"):
            for lib in (False, True):
                cases[f"lin_{name}_{kind}" + ("_cublas" if lib else "")] = (
                    lambda N=N, K=K, kind=kind, lib=lib: _linear_gemm_case(N, K, kind, lib))
    return cases


# (N, K) of the GENESIS-1B linears; M = 32768 tokens (8 sequences of 4096).
LINEAR_SHAPES = {"qkv": (6144, 2048), "o": (2048, 2048), "upgate": (11264, 2048), "down": (2048, 5632),
                 "head": (32000, 2048)}
LINEAR_TOKENS = 32768


def _linear_gemm_case(N: int, K: int, kind: str, lib: bool):
    """One of the three GEMMs of a linear layer y = x W^T at the training shape,
    on the CTA-pair kernel or through torch.matmul (cuBLAS)."""
    from llm_research_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad

    T = LINEAR_TOKENS
    x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    dy = torch.randn(T, N, device="cuda", dtype=torch.bfloat16)
    flops = 2.0 * T * N * K
    if kind == "fwd":
        out = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
        fn = (lambda: torch.matmul(x, w.t(), out=out)) if lib else (lambda: linear_fwd(x, w, out=out))
    elif kind == "dgrad":
        out = torch.empty(T, K, device="cuda", dtype=torch.bfloat16)
        fn = (lambda: torch.matmul(dy, w, out=out)) if lib else (lambda: linear_dgrad(dy, w, out=out))
    else:
        out = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        fn = (lambda: torch.matmul(dy.t(), x, out=out)) if lib else (lambda: linear_wgrad(dy, x, out=out))
    return fn, flops, 0.0


def _swiglu_up_case():
    """The fused SwiGLU up / gate projection (u, g and h = silu(g) * u from one
    CTA-pair launch) at the training shape; FLOPs of the two projections."""
    from llm_research_b200._ext import native

    T, (N2, K) = LINEAR_TOKENS, LINEAR_SHAPES["upgate"]
    F = N2 // 2
    x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
    w1 = torch.randn(F, K, device="cuda", dtype=torch.bfloat16) * 0.02
    wg = torch.randn(F, K, device="cuda", dtype=torch.bfloat16) * 0.02
    gu = torch.empty(T, 2 * F, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
    C = native()
    return (lambda: C.gemm_pair_swiglu(x, w1, wg, gu, h)), 2.0 * T * N2 * K, 0.0


def _qkv_rope_case():
    """The fused QKV projection with RoPE on the query and key heads (16 + 2 x 16
    heads of 128) at the training shape, sequences of 4096."""
    from llm_research_b200._ext import native

    T, (N, K) = LINEAR_TOKENS, LINEAR_SHAPES["qkv"]
    S, D = 4096, 128
    x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    out = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = torch.outer(torch.arange(S, device="cuda", dtype=torch.float32), inv)
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos().t().contiguous(), emb.sin().t().contiguous()  # column-major (128, S)
    C = native()
    return (lambda: C.gemm_pair_rope(x, w, out, cos, sin, S, 0, 2 * N // 3)), 2.0 * T * N * K, 0.0


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("names", nargs="*")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    peaks = _peaks()
    cases = _cases()
    timer = _Timer(args.warmup, args.iters)
    for name in args.names or list(cases):
        fn, flops, nbytes = cases[name]()
        ms = timer(fn)
        rec = {"case": name, "ms": round(ms, 4)}
        if flops:
            tf = flops / ms / 1e9
            rec.update(tflops=round(tf, 1), frac_of_measured_bf16=round(tf / peaks["bf16_tflops"], 3))
        if nbytes:
            gbs = nbytes / ms / 1e6
            rec.update(gbs=round(gbs, 1), frac_of_measured_hbm=round(gbs / peaks["hbm_gbs"], 3))
        rec["peaks"] = peaks["source"]
        print(json.dumps(rec), flush=True)
        del fn
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
