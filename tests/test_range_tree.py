"""Host range coding over bisection masses (the coder the decode loop runs):
symbols drawn from random distributions survive encode -> decode through the
library's RangeEncoder / RangeDecoder with the heap masses the softmax kernel
emits (left child of node 2^d - 1 + k = the first half of its aligned range)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import tsac_cuda


def heap_masses(p):
    """Left-child masses [1023] of a 1024-entry distribution, heap order."""
    out = np.zeros(1023, np.float32)
    for depth in range(10):
        width = 1024 >> depth
        for k in range(1 << depth):
            lo = k * width
            out[(1 << depth) - 1 + k] = np.float32(p[lo:lo + width // 2].sum(dtype=np.float64))
    return out


def random_rows(rng, count):
    masses = np.zeros((count, 1023), np.float32)
    symbols = np.zeros(count, np.uint16)
    for i in range(count):
        p = rng.dirichlet(np.full(1024, rng.choice([0.02, 0.3, 5.0])))
        masses[i] = heap_masses(p)
        symbols[i] = rng.choice(1024, p=p)
    return masses, symbols


def encode(masses, symbols):
    lib = tsac_cuda.library()
    out, size = ctypes.c_void_p(), ctypes.c_size_t()
    tsac_cuda.check(lib.tsac_cuda_range_encode_tree(masses.ctypes.data_as(ctypes.c_void_p),
                                                    symbols.ctypes.data_as(ctypes.c_void_p),
                                                    ctypes.c_size_t(len(symbols)), ctypes.byref(out),
                                                    ctypes.byref(size)))
    data = ctypes.string_at(out, size.value)
    lib.tsac_cuda_free(out)
    return data


def decode(stream, masses):
    lib = tsac_cuda.library()
    got = np.zeros(len(masses), np.uint16)
    buf = ctypes.create_string_buffer(stream, len(stream))
    tsac_cuda.check(lib.tsac_cuda_range_decode_tree(buf, ctypes.c_size_t(len(stream)),
                                                    masses.ctypes.data_as(ctypes.c_void_p),
                                                    ctypes.c_size_t(len(masses)),
                                                    got.ctypes.data_as(ctypes.c_void_p)))
    return got


@pytest.mark.parametrize("seed,count", [(0, 1), (1, 40), (2, 200)])
def test_round_trip(seed, count):
    rng = np.random.default_rng(seed)
    masses, symbols = random_rows(rng, count)
    stream = encode(masses, symbols)
    assert np.array_equal(decode(stream, masses), symbols)


def test_extreme_symbols_round_trip():
    """Improbable symbols (Q15 clamped to 1 or 32767 on the path) and both ends
    of the alphabet."""
    rng = np.random.default_rng(3)
    p = np.full(1024, 1e-9)
    p[500] = 1.0
    p /= p.sum()
    masses = np.repeat(heap_masses(p)[None], 6, axis=0)
    symbols = np.array([0, 1023, 500, 7, 500, 1022], np.uint16)
    assert np.array_equal(decode(encode(masses, symbols), masses), symbols)
    assert len(encode(masses, symbols[2:3])) < len(encode(masses, symbols[:1]))


def test_symbol_outside_alphabet_rejected():
    masses = np.zeros((1, 1023), np.float32)
    with pytest.raises(tsac_cuda.TsacError, match="alphabet"):
        encode(masses, np.array([1024], np.uint16))


def test_host_coder_matches_reference_encode_categorical():
    """The library's host coder over heap masses built with the reference's
    probability_sum (the oracle's restatement, pinned separately) writes the
    same bytes as the reference's own encode_categorical over the
    probabilities, and decodes that stream back."""
    from support import oracle, ptr, ref, ref_check

    rng = np.random.default_rng(7)
    count = 24
    probabilities = np.zeros((count, 1024), np.float32)
    symbols = np.zeros(count, np.uint16)
    for i in range(count):
        logits = rng.standard_normal(1024) * rng.choice([0.5, 3.0, 12.0])
        p = np.exp(logits - logits.max())
        p = (p / p.sum()).astype(np.float32)
        p[rng.random(1024) < 0.02] = np.float32(1e-41)  # subnormals exercise the FTZ sums
        probabilities[i] = p
        symbols[i] = rng.choice(1024, p=p.astype(np.float64) / p.astype(np.float64).sum())
    symbols[0], symbols[1] = 0, 1023
    lib = oracle()
    masses = np.zeros((count, 1023), np.float32)
    for i in range(count):
        row = probabilities[i]
        for depth in range(10):
            width = 1024 >> depth
            for k in range(1 << depth):
                left = np.ascontiguousarray(row[k * width:k * width + width // 2])
                masses[i, (1 << depth) - 1 + k] = lib.oracle_probability_sum(ptr(left), left.size)
    out, size = ctypes.c_void_p(), ctypes.c_size_t()
    ref_check(ref().ref_encode_categorical(ptr(probabilities), ptr(symbols), ctypes.c_size_t(count),
                                           ctypes.byref(out), ctypes.byref(size)))
    reference_stream = ctypes.string_at(out, size.value)
    ref().ref_free(out)
    assert encode(masses, symbols) == reference_stream
    assert np.array_equal(decode(reference_stream, masses), symbols)


def test_long_stream_matches_reference_byte_for_byte():
    """Thousands of symbols from very skewed and flat distributions: long runs
    of 0xff bytes and carries into them occur many times, and the library's
    coder (carry added into bytes already written) writes exactly the bytes
    of the reference's encode_categorical (pending-byte carry handling)."""
    from support import oracle, ptr, ref, ref_check

    rng = np.random.default_rng(11)
    count = 3000
    probabilities = np.zeros((count, 1024), np.float32)
    symbols = np.zeros(count, np.uint16)
    for i in range(count):
        p = rng.dirichlet(np.full(1024, rng.choice([0.005, 0.05, 1.0, 50.0])))
        p = np.maximum(p, 1e-30).astype(np.float32)
        probabilities[i] = p
        # Mostly likely symbols, sometimes a very unlikely one (long codes).
        symbols[i] = rng.integers(0, 1024) if rng.random() < 0.15 else int(np.argmax(p))
    masses = np.zeros((count, 1023), np.float32)
    oracle().oracle_bisection_masses(ptr(probabilities), ctypes.c_size_t(count), ptr(masses))
    out, size = ctypes.c_void_p(), ctypes.c_size_t()
    ref_check(ref().ref_encode_categorical(ptr(probabilities), ptr(symbols), ctypes.c_size_t(count),
                                           ctypes.byref(out), ctypes.byref(size)))
    reference_stream = ctypes.string_at(out, size.value)
    ref().ref_free(out)
    ours = encode(masses, symbols)
    assert len(ours) == len(reference_stream) and ours == reference_stream
    assert np.array_equal(decode(reference_stream, masses), symbols)
    # The stream holds runs of 0xff bytes (the bytes a later carry can reach).
    assert reference_stream.count(b"\xff\xff") > 0
