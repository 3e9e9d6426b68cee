"""Hot operations of the framework.

Every op has two implementations chosen by the device of its inputs:

* CUDA tensors run the hand-written sm_100a kernels of ``llm_research_b200._C``
  (the op raises if the extension is missing -- there is no silent fallback);
* CPU tensors run a plain PyTorch statement of the same math, which is also
  the numerical oracle the GPU tests compare against.
"""

from llm_research_b200.ops.norm import rms_norm, rms_norm_residual
from llm_research_b200.ops.activation import swiglu
from llm_research_b200.ops.rope import rope_qkv
from llm_research_b200.ops.attention import attention
from llm_research_b200.ops.loss import cross_entropy
from llm_research_b200.ops.routing import softmax_topk, chunk_mean_pool, compact_chunks, compact_chunks_fixed, route_slots
from llm_research_b200.ops.optim import muon_prologue, muon_prologue_into, muon_epilogue, newton_schulz, adamw_step, axpy_list
from llm_research_b200.ops.quant import int4_quantize, int4_dequantize, nvfp4_quantize, nvfp4_dequantize

__all__ = [
    "rms_norm", "rms_norm_residual", "swiglu", "rope_qkv", "attention", "cross_entropy",
    "softmax_topk", "chunk_mean_pool", "compact_chunks", "compact_chunks_fixed", "route_slots",
    "muon_prologue", "muon_prologue_into", "muon_epilogue", "newton_schulz", "adamw_step", "axpy_list",
    "int4_quantize", "int4_dequantize", "nvfp4_quantize", "nvfp4_dequantize",
]
