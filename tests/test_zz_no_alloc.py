"""The allocation-free prefix sum (bsx_prefix_sum_u32_noalloc).

It exists for callers that cannot allocate GPU memory (a foreign memory pool,
a real-time loop that cannot take cudaMalloc's synchronisation, a host that
does not let a plugin create a context). It must give the same result as the
regular bsx_prefix_sum_u32, call after call, although every call reuses the
same fixed device array. This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _regular(lib, x):
    h = C.c_void_p()
    assert lib.bsx_create(torch.cuda.current_device(), C.byref(h)) == 0
    try:
        out = torch.empty_like(x)
        assert lib.bsx_set_stream(h, C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        assert lib.bsx_prefix_sum_u32(h, C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(out.data_ptr())) == 0
        torch.cuda.synchronize()
        return out
    finally:
        lib.bsx_destroy(h)


def _noalloc(lib, x):
    out = torch.empty_like(x)
    st = lib.bsx_prefix_sum_u32_noalloc(C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(out.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    return out


def test_noalloc_prefix_sum_matches_regular_two_calls_in_a_row(cuda, bsx_lib):
    lib = bsx_lib.lib()
    g = torch.Generator(device="cuda")
    g.manual_seed(123)
    # two different inputs back to back: the shared scratch must be reset by each call
    for n in (5_000_011, 777):
        x = torch.randint(0, 1 << 20, (n,), generator=g, device="cuda", dtype=torch.int32)
        a = _noalloc(lib, x)
        b = _regular(lib, x)
        assert torch.equal(a, b), n
        ref = np.cumsum(x.cpu().numpy().view(np.uint32).astype(np.uint64)).astype(np.uint32)
        assert (a.cpu().numpy().view(np.uint32) == ref).all()


def test_noalloc_prefix_sum_rejects_sizes_beyond_its_limit(cuda, bsx_lib):
    lib = bsx_lib.lib()
    limit = 16_769_024
    x = torch.zeros(limit + 1, dtype=torch.int32, device="cuda")
    out = torch.empty_like(x)
    st = lib.bsx_prefix_sum_u32_noalloc(C.c_void_p(x.data_ptr()), limit + 1, C.c_void_p(out.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 3  # BSX_ERR_CAPACITY
    y = torch.ones(limit, dtype=torch.int32, device="cuda")
    r = _noalloc(lib, y)
    assert int(r[-1].item()) == limit
