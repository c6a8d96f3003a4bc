"""Pins the oracle (oracle/oracle.c) before anything is checked against it.

1. The reference's own known-answer tests, restated against the oracle:
   tests/numeric.cpp:60-76 (exhaustive BF16 rule), tests/scalar.cpp:35-53
   (convolution and BF8L KATs), tests/attention.cpp:87-104 (FNV checksum
   15737425383056432415 over 480 attention geometries).
2. Randomised cross-checks of every oracle function against the reference
   scalar path itself (oracle/_ref, built from the reference's sources).
"""
import ctypes

import numpy as np
import pytest

from support import bf16, c_size_t, f32, oracle, ptr, ref, ref_check


def test_bf16_rule_exhaustive():
    lib = oracle()
    upper = np.arange(65536, dtype=np.uint32)
    assert np.array_equal(f32(upper.astype(np.uint16)).view(np.uint32), upper << 16)
    for lower in (0, 0x7FFE, 0x7FFF, 0x8000, 0x8001, 0xFFFF):
        bits = (upper << 16) | lower
        expected = (upper + ((lower > 0x8000) | ((lower == 0x8000) & (upper & 1).astype(bool)))
                    ).astype(np.uint16)
        got = bf16(bits.view(np.float32))
        assert np.array_equal(got, expected)
        # The C oracle agrees with the rule on a stride through all patterns.
        for u in range(0, 65536, 251):
            assert lib.oracle_bf16(ctypes.c_float(bits.view(np.float32)[u])) == expected[u]


def test_bf8l_known_answer():
    x = np.zeros(256, np.float32)
    x[:4] = [127, 0.5, 1.5, -1.5]
    q = np.zeros(256, np.int8)
    s = np.zeros(1, np.uint16)
    oracle().oracle_bf8l(ptr(x), 256, ptr(q), ptr(s))
    assert s[0] == bf16(np.float32(1.0)) and list(q[:4]) == [127, 0, 2, -2]


def test_convolution_known_answers():
    lib = oracle()
    x = np.array([1, 2, 3], np.float32)
    w = np.array([2, 3], np.float32)
    b = np.array([1], np.float32)
    y = np.zeros(8, np.float32)
    n = lib.oracle_conv1d(1, 1, 2, 1, 0, 1, 0, ptr(w), ptr(b), ptr(x), 3, ptr(y))
    assert list(y[:n]) == [9, 14]
    n = lib.oracle_conv1d(1, 1, 2, 2, 0, 1, 1, ptr(w), ptr(b), ptr(x), 3, ptr(y))
    assert list(y[:n]) == [3, 4, 5, 7, 7, 10]


def _fnv(checksum, values):
    for v in values.tolist():
        checksum = ((checksum ^ (v & 255)) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        checksum = ((checksum ^ (v >> 8)) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return checksum


def test_attention_checksum():
    lib = oracle()
    checksum = 14695981039346656037
    for heads in (1, 2, 4):
        for coords in (3, 4, 7, 16, 128):
            for frames in (1, 3, 4, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 257):
                width = heads * coords
                i = np.arange(width)
                q = bf16(((i * 37 + 19) % 257 - 128).astype(np.float32) / np.float32(128))
                j = np.arange(frames * width)
                k = bf16(((j * 73 + j // 17) % 257 - 128).astype(np.float32) / np.float32(64))
                v = bf16(((j * 31 + j // 7) % 127 - 63).astype(np.float32) / np.float32(32))
                for prefill in (0, 1):
                    out = np.zeros(width, np.uint16)
                    lib.oracle_attention(ptr(q), ptr(k), ptr(v), heads, coords, frames, prefill,
                                         ptr(out))
                    checksum = _fnv(checksum, out)
    assert checksum == 15737425383056432415


# ---------------------------------------------------------------- vs _ref --
rng = np.random.default_rng(1234)


def _bf16_normal(*shape, scale=1.0):
    return bf16((rng.standard_normal(shape) * scale).astype(np.float32))


def test_exp_sum_q15_match_reference():
    lib, r = oracle(), ref()
    zs = np.concatenate([rng.uniform(-100, 100, 4000), [0.0, -0.0, 87.0, -88.0, 1e-40]]).astype(np.float32)
    for z in zs:
        assert np.float32(lib.oracle_exp(z)).view(np.uint32) == np.float32(r.ref_original_exp(z)).view(np.uint32)
    for n in (1, 2, 5, 8, 9, 63, 64, 65, 127, 128, 200, 511, 512, 1000, 1024):
        x = (rng.random(n) ** 8).astype(np.float32)
        x[rng.random(n) < 0.05] = np.float32(1e-41)  # subnormals exercise FTZ
        a = np.float32(lib.oracle_probability_sum(ptr(x), n))
        b = np.float32(r.ref_probability_sum(ptr(x), n))
        assert a.view(np.uint32) == b.view(np.uint32)
    for _ in range(2000):
        left, mass = np.float32(rng.random() ** 3), np.float32(rng.random() + 1e-3)
        assert lib.oracle_conditional_q15(left, mass) == r.ref_conditional_q15(left, mass)


def test_gelu_all_bf16_patterns_match_reference():
    lib, r = oracle(), ref()
    for v in range(0, 65536, 7):
        assert lib.oracle_gelu(v) == r.ref_gelu(v), v


@pytest.mark.parametrize("k,n,m", [(512, 64, 1), (512, 1536, 3), (2048, 512, 5), (1024, 512, 2)])
def test_linear_matches_reference(k, n, m):
    w = rng.integers(-128, 128, size=(n, k), dtype=np.int8)
    ws = (rng.uniform(0.5, 2.0, size=(k // 256, n)) / 127).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32)
    x = _bf16_normal(m, k)
    y0, y1 = np.zeros((m, n), np.uint16), np.zeros((m, n), np.uint16)
    oracle().oracle_linear(ptr(w), ptr(ws), ptr(b), k, n, ptr(x), m, ptr(y0))
    ref_check(ref().ref_packed_linear(ptr(w), ptr(ws), ptr(b), c_size_t(k), c_size_t(n), ptr(x),
                                      c_size_t(m), ptr(y1)))
    assert np.array_equal(y0, y1)


@pytest.mark.parametrize("time,prefill", [(1, 0), (12, 0), (64, 0), (65, 0), (200, 1), (1024, 0), (300, 1)])
def test_attention_matches_reference(time, prefill):
    q = _bf16_normal(512)
    k = _bf16_normal(time, 512)
    v = _bf16_normal(time, 512)
    y0, y1 = np.zeros(512, np.uint16), np.zeros(512, np.uint16)
    oracle().oracle_attention(ptr(q), ptr(k), ptr(v), 4, 128, time, prefill, ptr(y0))
    ref_check(ref().ref_attention(ptr(q), ptr(k), ptr(v), c_size_t(4), c_size_t(128), c_size_t(time),
                                  prefill, ptr(y1)))
    assert np.array_equal(y0, y1)


def test_norm_rotary_softmax_match_reference():
    lib, r = oracle(), ref()
    for scale in (1e-3, 1.0, 30.0):
        x = _bf16_normal(512, scale=scale)
        g = _bf16_normal(512, scale=0.1) + 0
        g = bf16(1 + f32(g))
        b = _bf16_normal(512, scale=0.05)
        y0, y1 = np.zeros(512, np.uint16), np.zeros(512, np.uint16)
        lib.oracle_layer_norm(ptr(x), ptr(g), ptr(b), 512, ptr(y0))
        ref_check(r.ref_layer_norm(ptr(x), ptr(g), ptr(b), c_size_t(512), ptr(y1)))
        assert np.array_equal(y0, y1)
        c = _bf16_normal(128)
        lib.oracle_rotary(ptr(x), ptr(c), 128, ptr(y0))
        ref_check(r.ref_rotary(ptr(x), ptr(c), c_size_t(128), ptr(y1)))
        assert np.array_equal(y0[:128], y1[:128])
        logits = _bf16_normal(1024, scale=scale * 3)
        s0, s1 = np.zeros(1024, np.uint16), np.zeros(1024, np.uint16)
        lib.oracle_softmax(ptr(logits), 1024, ptr(s0))
        ref_check(r.ref_softmax(ptr(logits), c_size_t(1024), ptr(s1)))
        assert np.array_equal(s0, s1)


@pytest.mark.parametrize("cin,cout,k,stride,dil,transposed,frames", [
    (3, 5, 7, 1, 1, 0, 40), (4, 6, 7, 1, 9, 0, 50), (8, 16, 4, 2, 1, 0, 33), (6, 3, 16, 8, 1, 0, 70),
    (5, 4, 16, 8, 1, 1, 9), (6, 3, 4, 2, 1, 1, 13), (2, 7, 3, 1, 1, 0, 5), (4, 4, 1, 1, 1, 0, 11)])
def test_conv1d_matches_reference(cin, cout, k, stride, dil, transposed, frames):
    pad = (k - 1) * dil // 2 if stride == 1 else (stride + 1) // 2
    w = rng.standard_normal(cin * cout * k).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    x = rng.standard_normal(frames * cin).astype(np.float32)
    y0 = np.zeros(100000, np.float32)
    y1 = np.zeros(100000, np.float32)
    n0 = oracle().oracle_conv1d(cin, cout, k, stride, pad, dil, transposed, ptr(w), ptr(b), ptr(x),
                                frames, ptr(y0))
    n1 = ctypes.c_size_t()
    ref_check(ref().ref_conv1d(c_size_t(cin), c_size_t(cout), c_size_t(k), c_size_t(stride),
                               c_size_t(pad), c_size_t(dil), transposed, ptr(w), ptr(b), ptr(x),
                               c_size_t(frames), ptr(y1), ctypes.byref(n1)))
    assert n0 == n1.value
    assert np.array_equal(y0[: n0 * cout].view(np.uint32), y1[: n0 * cout].view(np.uint32))


def test_snake_matches_reference():
    channels, frames = 24, 300
    x = (rng.standard_normal(channels * frames) * np.repeat(10.0 ** rng.uniform(-3, 4, frames), channels)
         ).astype(np.float32)
    a = rng.uniform(0.5, 1.5, channels).astype(np.float32)
    y0, y1 = np.zeros_like(x), np.zeros_like(x)
    oracle().oracle_snake(ptr(x), channels, frames, ptr(a), ptr(y0))
    ref_check(ref().ref_snake(ptr(x), c_size_t(channels), c_size_t(frames), ptr(a), ptr(y1)))
    assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32))


def test_rvq_nearest_and_projection_match_reference():
    """nearest_rvq_index (normalised query, ordered 8-FMA similarities, strict >
    so the lowest index wins ties) and the fused codebook projection."""
    lib_o, lib_r = oracle(), ref()
    lib_o.oracle_rvq_nearest.restype = ctypes.c_uint16
    lib_r.ref_rvq_nearest.restype = ctypes.c_uint16
    search = rng.standard_normal((1024, 8)).astype(np.float32)
    search /= np.linalg.norm(search, axis=1, keepdims=True)
    search[900] = search[5]  # an exact tie: index 5 must win
    queries = [rng.standard_normal(8).astype(np.float32) * s for s in (1e-3, 1.0, 40.0)]
    queries += [search[5] * np.float32(3.0), np.zeros(8, np.float32), search[1023].copy()]
    for q in queries:
        q = np.ascontiguousarray(q, dtype=np.float32)
        want = lib_r.ref_rvq_nearest(ptr(q), ptr(search))
        assert lib_o.oracle_rvq_nearest(ptr(q), ptr(search)) == want
    assert lib_r.ref_rvq_nearest(ptr(np.ascontiguousarray(search[5] * np.float32(3.0))), ptr(search)) == 5
    codebook = rng.standard_normal((1024, 8)).astype(np.float32)
    weights = (rng.standard_normal((1024, 8)) / 3).astype(np.float32)
    bias = (rng.standard_normal(1024) * 0.1).astype(np.float32)
    for index in (0, 17, 1023):
        y0, y1 = np.zeros(1024, np.float32), np.zeros(1024, np.float32)
        lib_o.oracle_rvq_project(ctypes.c_uint16(index), ptr(codebook), ptr(weights), ptr(bias), ptr(y0))
        ref_check(lib_r.ref_rvq_project(ctypes.c_uint16(index), ptr(codebook), ptr(weights), ptr(bias), ptr(y1)))
        assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32))
