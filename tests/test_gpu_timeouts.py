"""Bounded device waits: a wait on a flag that nothing sets gives up after its
poll limit (about a second), records an error code the host reads, and leaves
the CUDA context usable.  One GPU, one process; no fault is raised."""

import time

import pytest
import torch


@pytest.mark.gpu
def test_flag_wait_times_out_and_reports_status():
    from llm_research_b200._ext import native

    C = native()
    flags = torch.zeros(4, dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    t0 = time.time()
    C.ep_flag_wait(flags, 2, 7, err)  # no kernel and no peer ever raises these flags
    torch.cuda.synchronize()
    waited = time.time() - t0
    code = int(err[0])
    assert code != 0, "the wait should have run out and recorded its code"
    assert waited < 60.0
    # the context is still usable
    x = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == float((1 << 20) * ((1 << 20) - 1) / 2)
    # flags that are set pass without an error
    err.zero_()
    C.ep_flag_set(flags[0:1], 7)
    C.ep_flag_set(flags[1:2], 7)
    C.ep_flag_wait(flags, 2, 7, err)
    torch.cuda.synchronize()
    assert int(err[0]) == 0
