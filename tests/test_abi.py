"""The C-ABI library loads on a host without a GPU, exports every entry point
that include/tsac_cuda.h declares, and fails loudly (a device status and a
message, never a CPU fallback) when a call needs a GPU that is absent."""
from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

import tsac_cuda

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tsac_cuda.h"


def declared_entry_points():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tsac_cuda_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_entry_points()
    assert len(names) >= 30
    for required in ("tsac_cuda_encode", "tsac_cuda_decode", "tsac_cuda_encode_batch",
                     "tsac_cuda_decode_batch", "tsac_cuda_qlinear", "tsac_cuda_conv1d",
                     "tsac_cuda_transformer_probabilities", "tsac_cuda_rvq_encode"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = tsac_cuda.library()
    missing = [n for n in declared_entry_points() if not hasattr(lib, n)]
    assert missing == []


def test_status_codes_match_header():
    text = HEADER.read_text()
    for name, value in (("TSAC_CUDA_OK", 0), ("TSAC_CUDA_ERROR", 1), ("TSAC_CUDA_ERROR_DEVICE", 2),
                        ("TSAC_CUDA_ERROR_NUMERIC", 3)):
        assert re.search(rf"\b{name}\s*=\s*{value}\b", text), name


def test_context_without_gpu_fails_loudly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = tsac_cuda.library()
    ctx = ctypes.c_void_p()
    status = lib.tsac_cuda_context_create(b"/nonexistent", 0, ctypes.byref(ctx))
    assert status != 0
    assert not ctx.value
    with pytest.raises(tsac_cuda.TsacError):
        tsac_cuda.check(status)


def test_kernel_entry_point_without_gpu_fails_loudly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = tsac_cuda.library()
    p = ctypes.c_void_p(16)
    status = lib.tsac_cuda_snake(p, ctypes.c_size_t(1), ctypes.c_size_t(1), p, p, p,
                                 ctypes.c_void_p(0))
    assert status == 2  # TSAC_CUDA_ERROR_DEVICE: no device, nothing computed on the host


def test_context_setters_reject_null_context():
    lib = tsac_cuda.library()
    assert lib.tsac_cuda_set_host_threads(None, ctypes.c_uint(4)) == 1  # TSAC_CUDA_ERROR
    assert b"null" in lib.tsac_cuda_last_error()
    assert lib.tsac_cuda_set_exact_synthesis(None, 1) == 1


def test_adopted_buffer_lives_as_long_as_its_arrays():
    """Decoded PCM comes back in a malloc'd buffer that the binding wraps
    without copying: the array and its views read it, and the buffer is
    released (tsac_cuda_free) once the last of them is collected."""
    import gc
    import weakref

    import numpy as np

    libc = ctypes.CDLL(None)
    libc.malloc.restype = ctypes.c_void_p
    libc.malloc.argtypes = [ctypes.c_size_t]
    count = 1000
    raw = libc.malloc(count * 4)
    assert raw
    source = np.arange(count, dtype=np.float32)
    ctypes.memmove(raw, source.ctypes.data, count * 4)
    freed = []
    arr = tsac_cuda._adopt(ctypes.c_void_p(raw), count, np.float32)
    assert arr.dtype == np.float32 and arr.shape == (count,) and arr.ctypes.data == raw
    assert np.array_equal(arr, source)
    # The finaliser the binding registered fires once the storage goes away.
    storage = arr.base
    weakref.finalize(storage, freed.append, True)
    view = arr.reshape(-1, 2)
    del arr, storage
    gc.collect()
    assert not freed and view[499, 1] == 999.0
    del view
    gc.collect()
    assert freed == [True]
