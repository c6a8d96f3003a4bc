"""The allocation-free quantized linear entry point (tsac_cuda_qlinear_noalloc).

It exists for callers that cannot allocate device memory (a service that
reserves all GPU memory at start-up and forbids later cudaMalloc, or a
real-time audio thread that must not wait on the driver's allocator); its
scratch is a fixed array inside the library.  This file is collected last so
that a run stopping at its first failure has already run every other test.

Checks, through the C ABI: two calls in a row give exactly the output of the
allocating entry point tsac_cuda_qlinear on the same inputs (bit-exact, the
tolerance of every quantized-linear test), the second call using a smaller
shape while the first call's contents are still in the shared array; and a
call beyond the fixed scratch size fails with a clear error.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402


def _bf16(x):
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def _case(k, n, m, seed):
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda")
    w = torch.from_numpy(rng.integers(-128, 128, size=(n, k), dtype=np.int8)).to(dev)
    s = torch.from_numpy((rng.uniform(0.5, 2.0, size=(k // 256, n)) / 127).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.normal(0, 0.1, n).astype(np.float32)).to(dev)
    x = torch.from_numpy(_bf16(rng.standard_normal((m, k))).view(np.int16)).to(dev)
    r = torch.from_numpy(_bf16(rng.standard_normal((m, n))).view(np.int16)).to(dev)
    return w, s, b, x, r


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _noalloc(w, s, b, x, residual):
    n, k = w.shape
    m = x.shape[0]
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsac_cuda.check(tsac_cuda.library().tsac_cuda_qlinear_noalloc(
        _ptr(w), _ptr(s), _ptr(b), ctypes.c_size_t(k), ctypes.c_size_t(n), _ptr(x),
        ctypes.c_size_t(m), _ptr(residual), _ptr(y), _ptr(err),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return y.cpu().numpy()


def _allocating(w, s, b, x, residual):
    n, k = w.shape
    m = x.shape[0]
    y = torch.empty((m, n), dtype=torch.int16, device="cuda")
    scratch = torch.empty(tsac_cuda.qlinear_scratch_bytes(m, k), dtype=torch.uint8, device="cuda")
    tsac_cuda.qlinear(w, s, b, x, y, scratch, residual=residual)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_on_two_calls_in_a_row():
    lib = tsac_cuda.library()
    lib.tsac_cuda_qlinear_noalloc_max_elements.restype = ctypes.c_size_t
    assert lib.tsac_cuda_qlinear_noalloc_max_elements() == 1 << 20
    first = _case(4096, 1024, 256, seed=1)          # fills the whole scratch
    second = _case(512, 1536, 3, seed=2)            # smaller: stale bytes remain
    for w, s, b, x, r in (first, second):
        for residual in (None, r):
            expected = _allocating(w, s, b, x, residual)
            got = _noalloc(w, s, b, x, residual)
            assert np.array_equal(got, expected)


def test_noalloc_rejects_calls_beyond_its_scratch():
    w, s, b, x, _ = _case(4096, 64, 257, seed=3)
    with pytest.raises(tsac_cuda.TsacError, match="exceeds its fixed 1 MiB scratch"):
        _noalloc(w, s, b, x, None)
