"""Allocation-free causal-conv backward, called through its exported C symbol.

``cqb_conv_bwd_noalloc`` is for callers that cannot allocate device memory during the call
(allocator hooks, C hosts without PyTorch, pre-sized memory pools). Its weight-gradient
partials live in a static device array instead of a fresh buffer. These tests compare it with
the tensor entry point ``conv_bwd`` on two calls in a row (the second call reuses the array that
the first one left behind), including an input that fills the array exactly, check that the
calls leave the device's free memory unchanged, and check that oversize or malformed inputs are
refused. The C prototypes are those of ``csrc/noalloc.h``.

The file name sorts last on purpose, so that a run stopping at its first failure has already
run every other test.
"""

import ctypes

import pytest
import torch

from cq_pretrain_b200.ops import _ext

pytestmark = pytest.mark.gpu


def _lib():
    assert _ext.cuda_kernels_enabled(), "the sm_100a library must be loaded"
    lib = ctypes.CDLL(str(_ext.library_path()))
    fn = lib.cqb_conv_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_long, ctypes.c_long, ctypes.c_void_p]
    lib.cqb_noalloc_last_error.restype = ctypes.c_char_p
    lib.cqb_conv_bwd_noalloc_scratch_floats.restype = ctypes.c_size_t
    return lib


@pytest.mark.parametrize("bounds,C", [((0, 300, 301, 777), 1024), ((0, 4096), 6144),
                                      ((0, 5000, 16384), 8192)])   # the last one fills the array exactly
def test_noalloc_conv_bwd_matches_tensor_entry(bounds, C):
    lib = _lib()
    torch.manual_seed(0)
    n = bounds[-1]
    x = torch.randn(n, C, device="cuda").to(torch.bfloat16)
    dy = torch.randn(n, C, device="cuda").to(torch.bfloat16)
    w = torch.rand(C, 4, device="cuda") - 0.5
    pos = torch.cat([torch.arange(b - a, dtype=torch.int32) for a, b in zip(bounds, bounds[1:])]).cuda()
    if C == 8192:
        assert -(-n // 256) * C * 4 == lib.cqb_conv_bwd_noalloc_scratch_floats()
    ref_dx, ref_dw = _ext.ops().conv_bwd(dy, x, w, pos)
    wT = w.t().contiguous()
    stream = torch.cuda.current_stream().cuda_stream
    outs = [(torch.empty_like(x), torch.empty(C, 4, device="cuda")) for _ in range(2)]
    for dx, dw in outs:
        dx.fill_(float("nan"))
        dw.fill_(float("nan"))
    torch.cuda.synchronize()
    free_before = None
    for dx, dw in outs:
        rc = lib.cqb_conv_bwd_noalloc(dy.data_ptr(), x.data_ptr(), wT.data_ptr(), pos.data_ptr(), dx.data_ptr(),
                                      dw.data_ptr(), n, C, stream)
        assert rc == 0, lib.cqb_noalloc_last_error()
        torch.cuda.synchronize()
        free_now = torch.cuda.mem_get_info()[0]
        if free_before is not None:   # the second call allocates nothing on the device
            assert free_now == free_before, (free_before, free_now)
        free_before = free_now
    for dx, dw in outs:
        torch.testing.assert_close(dx.float(), ref_dx.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dw, ref_dw, rtol=1e-4, atol=1e-4)


def test_noalloc_conv_bwd_rejects_oversize_and_bad_shapes():
    lib = _lib()
    limit = lib.cqb_conv_bwd_noalloc_scratch_floats()
    C = 8192
    n = (limit // (C * 4) + 1) * 256          # one 256-row block more than the array holds
    buf = torch.empty(16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    p = buf.data_ptr()
    # sizes are checked before any buffer is read, so small placeholders suffice here
    rc = lib.cqb_conv_bwd_noalloc(p, p, p, p, p, p, n, C, stream)
    assert rc == 2 and b"too large" in lib.cqb_noalloc_last_error()
    rc = lib.cqb_conv_bwd_noalloc(p, p, p, p, p, p, 4, 12, stream)
    assert rc == 1 and b"multiple of 8" in lib.cqb_noalloc_last_error()
