"""The allocation-free cross-entropy entry point agrees with the allocating one.

``tx_softmax_xent_fwd_noalloc`` serves callers that cannot allocate device memory
(a host runtime that reserves all of the GPU's memory for its own allocator, or
a latency-bound loop that cannot pay for the device-wide synchronisation of
cudaMalloc / cudaFree).  It is called here through the C ABI, twice in a row on
different inputs, and must give the same loss as ``tx_softmax_xent_fwd`` within
the 1e-5 relative tolerance the other cross-entropy tests use, without touching
the context allocator.  The file is named to run last, and it also passes on
its own in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_cross_entropy_matches_allocating_entry_point():
    import tynx_b200 as tx
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    lib = N.lib
    rng = np.random.default_rng(20)
    # two calls in a row: the second is smaller, so stale rows of the first call
    # in the shared array would change its result if they were read
    for rows, cols in [(4096, 10), (1000, 37)]:
        z = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
        y = rng.integers(0, cols, rows).astype(np.int64)
        Z, Y = tx.Tensor(z), tx.Tensor(y)
        want, got = tx.zeros(1), tx.zeros(1)
        ctx.check(lib.tx_softmax_xent_fwd(ctx.handle, Z.ptr, Y.ptr, rows, cols, want.ptr))
        tx.synchronize()
        in_use, cached = C.c_uint64(), C.c_uint64()
        lib.tx_mem_stats(ctx.handle, C.byref(in_use), C.byref(cached))
        before = (in_use.value, cached.value)
        ctx.check(lib.tx_softmax_xent_fwd_noalloc(ctx.handle, Z.ptr, Y.ptr, rows, cols, got.ptr))
        lib.tx_mem_stats(ctx.handle, C.byref(in_use), C.byref(cached))
        assert (in_use.value, cached.value) == before  # the context allocator was not used
        a, b = want.item(), got.item()
        assert abs(b - a) <= 1e-5 * max(1.0, abs(a)), (rows, a, b)

    # inputs above the stated maximum are rejected before any launch
    code = lib.tx_softmax_xent_fwd_noalloc(ctx.handle, Z.ptr, Y.ptr, (1 << 18) + 1, 37, got.ptr)
    assert code == N.TX_ERR_SHAPE
    buf = C.create_string_buffer(256)
    assert lib.tx_last_error(ctx.handle, buf, 256) == N.TX_ERR_SHAPE
    assert b"262144" in buf.value
