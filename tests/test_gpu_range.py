"""Device range decoding (the optional GPU-resident alternative to the host
decoders): several streams whose rows interleave, decoded over two calls so
the cursors carry the decoder state, give exactly the symbols the library's
host RangeEncoder coded; a payload whose code starts outside its interval
stops with status 1 and the range-error bit."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import tsac_cuda
from test_range_tree import encode, random_rows

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_device_decoder_matches_host_coder():
    import torch

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(11)
    counts = [1, 9, 40, 0, 17]
    per_stream = [random_rows(rng, c) for c in counts]
    payloads = [encode(m, s) for m, s in per_stream]
    payloads.append(b"\xff\xff\xff\x00")  # code 0xffffff >= 0xff0000: invalid from the start
    counts.append(3)
    per_stream.append((np.full((3, 1023), 0.5, np.float32), np.zeros(3, np.uint16)))
    streams = len(payloads)
    offsets = np.cumsum([0] + [len(p) for p in payloads[:-1]]).astype(np.int64)
    sizes = np.array([len(p) for p in payloads], np.int64)
    # Interleave rows round-robin over streams, each stream's rows in order.
    order, cursor = [], [0] * streams
    while any(cursor[s] < counts[s] for s in range(streams)):
        for s in range(streams):
            if cursor[s] < counts[s]:
                order.append((s, cursor[s]))
                cursor[s] += 1
    rows = np.array([s for s, _ in order], np.int32)
    masses = np.stack([per_stream[s][0][i] for s, i in order]).astype(np.float32)
    expected = np.array([per_stream[s][1][i] for s, i in order], np.uint16)

    lib = tsac_cuda.library()
    lib.tsac_cuda_range_cursor_bytes.restype = ctypes.c_size_t
    cursor_bytes = lib.tsac_cuda_range_cursor_bytes()
    d_bytes = torch.from_numpy(np.frombuffer(b"".join(payloads), np.uint8).copy()).to(dev)
    d_offsets = torch.from_numpy(offsets).to(dev)
    d_sizes = torch.from_numpy(sizes).to(dev)
    d_cursors = torch.zeros(streams * cursor_bytes, dtype=torch.uint8, device=dev)
    d_rows = torch.from_numpy(rows).to(dev)
    d_masses = torch.from_numpy(masses).to(dev)
    d_symbols = torch.full((len(rows),), -1, dtype=torch.int16, device=dev)
    d_error = torch.zeros(1, dtype=torch.int32, device=dev)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    tsac_cuda.check(lib.tsac_cuda_range_start(_ptr(d_bytes), _ptr(d_offsets), _ptr(d_sizes), _ptr(d_cursors),
                                              ctypes.c_size_t(streams), _ptr(d_error), s))
    half = len(rows) // 2
    for lo, hi in ((0, half), (half, len(rows))):
        tsac_cuda.check(lib.tsac_cuda_range_decode(
            _ptr(d_bytes), _ptr(d_offsets), _ptr(d_sizes), _ptr(d_cursors), ctypes.c_size_t(streams),
            ctypes.c_void_p(d_rows.data_ptr() + 4 * lo), ctypes.c_size_t(hi - lo),
            ctypes.c_void_p(d_masses.data_ptr() + 4 * 1023 * lo), ctypes.c_void_p(d_symbols.data_ptr() + 2 * lo),
            _ptr(d_error), s))
    torch.cuda.synchronize()
    got = d_symbols.cpu().numpy().view(np.uint16)
    bad = rows == streams - 1
    assert np.array_equal(got[~bad], expected[~bad])
    assert np.all(got[bad] == 0)
    status = d_cursors.cpu().numpy().view(np.uint32).reshape(streams, 4)[:, 3]
    assert list(status) == [0] * (streams - 1) + [1]
    assert int(d_error.item()) & 2
