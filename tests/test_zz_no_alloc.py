"""The allocation-free C entry point ``lrb_rmsnorm_bwd_bf16_noalloc``.

Called through ctypes from the extension's shared object and compared with the
``rmsnorm_bwd`` op of the same extension on two calls in a row (the second
call reuses the static scratch array the first one wrote).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

ERR_ARGS, ERR_TOO_LARGE = 1, 2
MAX_D = 6400


def _entry():
    from llm_research_b200._ext import native

    lib = ctypes.CDLL(native().__file__)
    fn = lib.lrb_rmsnorm_bwd_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_char_p,
                                          ctypes.c_int]
    return fn


def test_noalloc_rejects_oversized_rows_without_touching_the_device():
    fn = _entry()
    buf = ctypes.create_string_buffer(256)
    fake = 1 << 20  # 16-byte aligned, never dereferenced: the size check comes first
    rc = fn(fake, fake, fake, fake, None, fake, fake, 8, MAX_D + 1, None, buf, 256)
    assert rc == ERR_TOO_LARGE
    assert b"exceeds the maximum" in buf.value
    rc = fn(None, fake, fake, fake, None, fake, fake, 8, 64, None, buf, 256)
    assert rc == ERR_ARGS


@pytest.mark.gpu
@pytest.mark.parametrize("rows,d,with_ds", [(4099, 2048, False), (1000, 2048, True), (777, 1000, True),
                                            (64, 6400, False)])
def test_noalloc_matches_rmsnorm_bwd_twice(rows, d, with_ds):
    from llm_research_b200._ext import native

    C = native()
    fn = _entry()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(rows * 7 + d)
    x = torch.randn(rows, d, device=dev, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(d, device=dev, generator=g)).to(torch.bfloat16)
    _, rstd, _ = C.rmsnorm_fwd(x, w, 1e-6, None, torch.bfloat16)
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((d,), float("nan"), device=dev, dtype=torch.float32)
    buf = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        dy = torch.randn(rows, d, device=dev, generator=g).to(torch.bfloat16)
        ds = torch.randn(rows, d, device=dev, generator=g).to(torch.bfloat16) if with_ds else None
        dx_ref, dw_ref = C.rmsnorm_bwd(dy, x, w, rstd, ds)
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), ds.data_ptr() if with_ds else None,
                dx.data_ptr(), dw.data_ptr(), rows, d, stream, buf, 256)
        assert rc == 0, buf.value.decode()
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(dx.float(), dx_ref.float(), rtol=1e-2, atol=1e-2, msg=f"dx, call {call}")
        torch.testing.assert_close(dw, dw_ref, rtol=1e-4, atol=1e-3, msg=f"dw, call {call}")
