"""Allocation-free INT8 linear (h3b200_int8_linear_noalloc), called through the C ABI.

Some callers of this library cannot allocate device memory per call -- a host
runtime that owns all device memory and passes only inputs and outputs, or a
serving loop that must not allocate after start-up. For them the entry point
keeps its quantized-activation scratch in a static device array. This test
checks, on two calls in a row with different inputs, that its output is
identical to the workspace-based h3b200_int8_linear, and that a request larger
than the static scratch is refused with a clear error.

The file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

from h3b200 import _lib

pytestmark = pytest.mark.gpu


def _linear_with_workspace(lib, x, w, ws, stream, bias=None, act=0):
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    nbytes = int(lib.h3b200_int8_linear_workspace_bytes(m, k))
    work = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    rc = lib.h3b200_int8_linear(x.data_ptr(), x.stride(0), w.data_ptr(), ws.data_ptr(), ws.numel(),
                                None if bias is None else bias.data_ptr(), act, out.data_ptr(), m, n, k,
                                work.data_ptr(), nbytes, stream)
    assert rc == 0, lib.h3b200_last_error()
    return out


def _linear_noalloc(lib, x, w, ws, stream, bias=None, act=0):
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    rc = lib.h3b200_int8_linear_noalloc(x.data_ptr(), x.stride(0), w.data_ptr(), ws.data_ptr(), ws.numel(),
                                        None if bias is None else bias.data_ptr(), act, out.data_ptr(), m, n, k,
                                        stream)
    assert rc == 0, lib.h3b200_last_error()
    return out


def test_noalloc_matches_workspace_entry_point_two_calls():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator().manual_seed(77)
    w = torch.randint(-127, 128, (1024, 3072), generator=gen, dtype=torch.int16).to(torch.int8).cuda()
    ws = (torch.rand(1024, generator=gen) * 1e-3).cuda()
    for rows in (2048, 300):   # two calls in a row, different inputs and sizes
        x = torch.randn(rows, 3072, generator=gen).to(torch.bfloat16).cuda()
        ref = _linear_with_workspace(lib, x, w, ws, stream)
        got = _linear_noalloc(lib, x, w, ws, stream)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_noalloc_gelu_input_and_bias_match_workspace_entry_point():
    """tanh-GELU on the input and a bias in the epilogue, two calls in a row, bit for bit."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator().manual_seed(78)
    w = torch.randint(-127, 128, (512, 1024), generator=gen, dtype=torch.int16).to(torch.int8).cuda()
    ws = (torch.rand(512, generator=gen) * 1e-3).cuda()
    bias = (torch.randn(512, generator=gen) * 0.1).to(torch.bfloat16).cuda()
    for rows in (1000, 64):
        x = (torch.randn(rows, 1024, generator=gen) * 2).to(torch.bfloat16).cuda()
        ref = _linear_with_workspace(lib, x, w, ws, stream, bias, _lib.ACT_GELU_TANH)
        got = _linear_noalloc(lib, x, w, ws, stream, bias, _lib.ACT_GELU_TANH)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_noalloc_rejects_requests_beyond_the_static_scratch():
    lib = _lib.load()
    cap = int(lib.h3b200_int8_linear_noalloc_max_scratch_bytes())
    assert cap == 8 << 20
    k = 3072
    m = cap // k + 1
    rc = lib.h3b200_int8_linear_noalloc(ctypes.c_void_p(16), k, ctypes.c_void_p(16), ctypes.c_void_p(16), 1, None,
                                        0, ctypes.c_void_p(16), m, 256, k, None)
    assert rc == _lib.ERR_INVALID
    assert b"static scratch" in lib.h3b200_last_error()
