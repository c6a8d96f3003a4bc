"""DAC analysis/synthesis and RVQ kernels on the GPU vs the oracle and the reference.

Exact-order convolutions and Snake are bit-exact against the oracle's
restatement of scalar::Conv1d / scalar_snake_frames (pinned in test_oracle.py);
the whole DAC windows and RVQ are bit-exact against the reference scalar path
itself (oracle/_ref) on the seeded package.
"""
import ctypes

import numpy as np
import pytest

from support import c_size_t, oracle, ptr, ref, ref_available, ref_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _conv_gpu(x, w_ref, b, cin, cout, k, stride, pad, dil, transposed, residual=None):
    frames = x.shape[0]
    # Reference stored order -> device [tap][in][out].
    if transposed:
        w = w_ref.reshape(cin, k, cout).transpose(1, 0, 2)
    else:
        w = w_ref.reshape(cout, k, cin).transpose(1, 2, 0)
    span = (k - 1) * dil + 1
    out_frames = (frames - 1) * stride + span - 2 * pad if transposed else (frames + 2 * pad - span) // stride + 1
    lib = tsac_cuda.library()
    lib.tsac_cuda_conv1d_scratch_bytes.restype = ctypes.c_size_t
    nbytes = lib.tsac_cuda_conv1d_scratch_bytes(c_size_t(out_frames), stride, transposed)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    tx, tw, tb = _dev(x.astype(np.float32)), _dev(w.astype(np.float32)), _dev(b)
    ty = torch.empty((out_frames, cout), dtype=torch.float32, device="cuda")
    tr = _dev(residual) if residual is not None else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)  # noqa: E731
    tsac_cuda.check(lib.tsac_cuda_conv1d(dp(tx), c_size_t(frames), dp(tw), dp(tb), dp(tr), dp(ty),
                                         c_size_t(cin), c_size_t(cout), c_size_t(k), c_size_t(stride),
                                         c_size_t(pad), c_size_t(dil), transposed, dp(scratch),
                                         c_size_t(nbytes), dp(err),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return ty.cpu().numpy()


@pytest.mark.parametrize("cin,cout,k,stride,dil,transposed,frames", [
    (64, 64, 7, 1, 1, 0, 300), (64, 64, 7, 1, 9, 0, 200), (64, 64, 1, 1, 1, 0, 129),
    (128, 256, 8, 4, 1, 0, 513), (512, 1024, 16, 8, 1, 0, 64), (1024, 1024, 3, 1, 1, 0, 37),
    (2, 64, 7, 1, 1, 0, 1000), (40, 72, 7, 1, 3, 0, 3),
    (1536, 768, 16, 8, 1, 1, 11), (384, 192, 8, 4, 1, 1, 50), (192, 96, 4, 2, 1, 1, 133),
    (96, 2, 7, 1, 1, 0, 700), (96, 1, 7, 1, 1, 0, 65)])
def test_conv1d_bit_exact(cin, cout, k, stride, dil, transposed, frames):
    rng = np.random.default_rng(cin * 131 + cout + k + frames)
    pad = (k - 1) * dil // 2 if stride == 1 else (stride + 1) // 2
    w = (rng.standard_normal(cin * cout * k) / np.sqrt(cin * k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32) * np.float32(0.1)
    x = rng.standard_normal((frames, cin)).astype(np.float32)
    y = np.zeros(400000, np.float32)
    n = oracle().oracle_conv1d(cin, cout, k, stride, pad, dil, transposed, ptr(w), ptr(b), ptr(x),
                               frames, ptr(y))
    expected = y[: n * cout].reshape(n, cout)
    got = _conv_gpu(x, w, b, cin, cout, k, stride, pad, dil, transposed)
    assert got.shape == expected.shape
    bad = np.flatnonzero(got.view(np.uint32).ravel() != expected.view(np.uint32).ravel())
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}"


def _conv_f64(x, w_ref, b, cin, cout, k, stride, pad, dil, transposed):
    """float64 convolution with the reference's geometry (src/common/dsp.tpp:141-178)."""
    frames = x.shape[0]
    x = x.astype(np.float64)
    if transposed:
        w = w_ref.reshape(cin, k, cout).astype(np.float64)
        out_frames = (frames - 1) * stride + k - 2 * pad
        y = np.zeros((out_frames + 2 * pad + k, cout))
        for tap in range(k):
            y[tap: tap + (frames - 1) * stride + 1: stride] += x @ w[:, tap, :]
        y = y[pad: pad + out_frames]
    else:
        w = w_ref.reshape(cout, k, cin).astype(np.float64)
        out_frames = frames + 2 * pad - (k - 1) * dil
        xp = np.zeros((frames + 2 * pad, cin))
        xp[pad: pad + frames] = x
        y = np.zeros((out_frames, cout))
        for tap in range(k):
            y += xp[tap * dil: tap * dil + out_frames] @ w[:, tap, :].T
    return y + b.astype(np.float64)


def _conv_tensor(x, w_ref, b, cin, cout, k, stride, pad, dil, transposed, residual=None, alpha=None):
    frames = x.shape[0]
    if transposed:
        w = w_ref.reshape(cin, k, cout).transpose(1, 0, 2)
        out_frames = frames * stride
    else:
        w = w_ref.reshape(cout, k, cin).transpose(1, 2, 0)
        out_frames = frames
    lib = tsac_cuda.library()
    tx, tw, tb = _dev(x.astype(np.float32)), _dev(w.astype(np.float32)), _dev(b)
    ty = torch.empty((out_frames, cout), dtype=torch.float32, device="cuda")
    tr = _dev(residual) if residual is not None else None
    ta = _dev(alpha) if alpha is not None else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)  # noqa: E731
    tsac_cuda.check(lib.tsac_cuda_conv1d_tensor(
        dp(tx), c_size_t(frames), dp(tw), dp(tb), dp(tr), dp(ta), dp(ty), c_size_t(cin),
        c_size_t(cout), c_size_t(k), c_size_t(stride), c_size_t(pad), c_size_t(dil), transposed,
        dp(err), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return ty.cpu().numpy()


# Per-output bound for the 3xTF32 tensor-core convolution: |got - exact| <=
# 2^-17 * (sum |x||w| + |b|); the split keeps about 2^-20 per product.
TENSOR_REL = 2.0 ** -17


@pytest.mark.parametrize("cin,cout,k,stride,dil,transposed,frames", [
    (1024, 1536, 7, 1, 1, 0, 23), (768, 768, 7, 1, 9, 0, 300), (768, 768, 1, 1, 1, 0, 129),
    (384, 384, 7, 1, 3, 0, 517), (96, 96, 7, 1, 9, 0, 1000), (192, 192, 1, 1, 1, 0, 64),
    (1536, 768, 16, 8, 1, 1, 11), (768, 384, 16, 8, 1, 1, 40), (384, 192, 8, 4, 1, 1, 50),
    (192, 96, 4, 2, 1, 1, 133), (96, 96, 7, 1, 1, 0, 1)])
def test_conv1d_tensor_cores_accuracy(cin, cout, k, stride, dil, transposed, frames):
    rng = np.random.default_rng(cin * 7 + cout + k + frames)
    pad = (k - 1) * dil // 2 if not transposed else stride // 2
    w = (rng.standard_normal(cin * cout * k) / np.sqrt(cin * k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32) * np.float32(0.1)
    x = rng.standard_normal((frames, cin)).astype(np.float32)
    exact = _conv_f64(x, w, b, cin, cout, k, stride, pad, dil, transposed)
    scale = _conv_f64(np.abs(x), np.abs(w), np.abs(b), cin, cout, k, stride, pad, dil, transposed)
    got = _conv_tensor(x, w, b, cin, cout, k, stride, pad, dil, transposed)
    assert got.shape == exact.shape
    ratio = np.abs(got - exact) / scale
    assert ratio.max() <= TENSOR_REL, f"max error / sum|xw| = {ratio.max():.3g} (2^{np.log2(ratio.max()):.1f})"


def test_conv1d_tensor_cores_residual_and_snake():
    rng = np.random.default_rng(5)
    cin = cout = 192
    w = (rng.standard_normal(cin * cout * 7) / np.sqrt(cin * 7)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    x = rng.standard_normal((300, cin)).astype(np.float32)
    res = rng.standard_normal((300, cout)).astype(np.float32)
    a = rng.uniform(0.5, 1.5, cout).astype(np.float32)
    raw = _conv_tensor(x, w, b, cin, cout, 7, 1, 3, 1, 0, residual=res)
    exact = _conv_f64(x, w, b, cin, cout, 7, 1, 3, 1, 0) + res
    scale = _conv_f64(np.abs(x), np.abs(w), np.abs(b), cin, cout, 7, 1, 3, 1, 0) + np.abs(res)
    assert (np.abs(raw - exact) / scale).max() <= TENSOR_REL
    act = _conv_tensor(x, w, b, cin, cout, 7, 1, 3, 1, 0, residual=res, alpha=a)
    expected = np.zeros_like(raw)
    oracle().oracle_snake(ptr(np.ascontiguousarray(raw)), cout, 300, ptr(a), ptr(expected))
    # The tensor path multiplies sin^2 by a precomputed 1 / (alpha + eps)
    # instead of dividing: one extra rounding of a quotient <= 2 (alpha >= 0.5),
    # then the same final add.
    assert (np.abs(act.astype(np.float64) - expected) <= 2.0 ** -21 * (1.0 + np.abs(expected))).all()


def test_conv1d_residual_epilogue():
    rng = np.random.default_rng(3)
    cin = cout = 64
    w = (rng.standard_normal(cin * cout) / 8).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    x = rng.standard_normal((77, cin)).astype(np.float32)
    res = rng.standard_normal((77, cout)).astype(np.float32)
    y = np.zeros(77 * cout, np.float32)
    oracle().oracle_conv1d(cin, cout, 1, 1, 0, 1, 0, ptr(w), ptr(b), ptr(x), 77, ptr(y))
    expected = res + y.reshape(77, cout)
    got = _conv_gpu(x, w, b, cin, cout, 1, 1, 0, 1, 0, residual=res)
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))


def test_snake_bit_exact():
    rng = np.random.default_rng(11)
    channels, frames = 96, 4000
    scale = np.repeat(10.0 ** rng.uniform(-4, 5, frames), channels)
    x = (rng.standard_normal(channels * frames) * scale).astype(np.float32)
    a = rng.uniform(0.5, 1.5, channels).astype(np.float32)
    expected = np.zeros_like(x)
    oracle().oracle_snake(ptr(x), channels, frames, ptr(a), ptr(expected))
    tx, ta = _dev(x), _dev(a)
    ty = torch.empty_like(tx)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    tsac_cuda.check(tsac_cuda.library().tsac_cuda_snake(
        dp(tx), c_size_t(channels), c_size_t(frames), dp(ta), dp(ty), dp(err),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(ty.cpu().numpy().view(np.uint32), expected.view(np.uint32))


# ------------------------------------------------------- model-level (seeded)
@pytest.fixture(scope="module")
def package():
    return tsac_cuda.seeded_package(0)


@pytest.fixture(scope="module")
def analyzer(package):
    a = tsac_cuda.CudaAnalyzer(package, 0)
    yield a
    a.close()


@pytest.mark.parametrize("channels,frames", [(2, 12), (1, 9)])
def test_dac_analysis_window_matches_reference(analyzer, package, channels, frames):
    if not ref_available():
        pytest.skip("reference oracle not built")
    pcm = synthetic.music_like(21 + channels, frames * 512 / 44100.0, channels)
    pcm = pcm[: frames * 512]
    got = analyzer.dac_analysis(channels, pcm)
    expected = np.zeros((frames, 1024), np.float32)
    ref_check(ref().ref_dac_analysis(str(package).encode(), channels, ptr(pcm),
                                     c_size_t(frames * 512), ptr(expected)))
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))


@pytest.mark.parametrize("channels,frames", [(2, 3), (1, 2)])
def test_dac_synthesis_window_matches_reference(analyzer, package, channels, frames):
    if not ref_available():
        pytest.skip("reference oracle not built")
    rng = np.random.default_rng(channels + frames)
    tokens = rng.integers(0, 1024, (frames, 12 if channels == 2 else 9)).astype(np.uint16)
    latent = analyzer.rvq_decode(channels, tokens.shape[1], tokens)
    analyzer.set_exact_synthesis(True)
    try:
        got = analyzer.dac_synthesis(channels, latent)
    finally:
        analyzer.set_exact_synthesis(False)
    expected = np.zeros((frames * 512, channels), np.float32)
    ref_check(ref().ref_dac_synthesis(str(package).encode(), channels, ptr(latent),
                                      c_size_t(frames), ptr(expected)))
    bad = np.flatnonzero(got.view(np.uint32).ravel() != expected.view(np.uint32).ravel())
    assert bad.size == 0, f"{bad.size} of {got.size} differ; max |d| {np.abs(got - expected).max()}"


@pytest.mark.parametrize("channels,frames", [(2, 3), (1, 2), (2, 17)])
def test_dac_synthesis_tensor_cores_within_tolerance(analyzer, package, channels, frames):
    """3xTF32 tcgen05 synthesis vs the reference: |a - b| <= 1e-4 (1 + max(|a|, |b|)),
    the reference's own pipeline tolerance (tests/metal_optimized.cpp:741-745)."""
    if not ref_available():
        pytest.skip("reference oracle not built")
    rng = np.random.default_rng(100 + channels + frames)
    tokens = rng.integers(0, 1024, (frames, 12 if channels == 2 else 9)).astype(np.uint16)
    latent = analyzer.rvq_decode(channels, tokens.shape[1], tokens)
    got = analyzer.dac_synthesis(channels, latent).astype(np.float64)
    expected = np.zeros((frames * 512, channels), np.float32)
    ref_check(ref().ref_dac_synthesis(str(package).encode(), channels, ptr(latent),
                                      c_size_t(frames), ptr(expected)))
    expected = expected.astype(np.float64)
    bound = 1e-4 * (1.0 + np.maximum(np.abs(got), np.abs(expected)))
    excess = np.abs(got - expected) - bound
    assert excess.max() <= 0, f"max |d| {np.abs(got - expected).max():.3g}"


@pytest.mark.parametrize("channels,books", [(2, 12), (2, 5), (1, 9)])
def test_rvq_encode_decode_match_reference(analyzer, package, channels, books):
    if not ref_available():
        pytest.skip("reference oracle not built")
    rng = np.random.default_rng(books)
    latent = (rng.standard_normal((57, 1024)) * 2).astype(np.float32)
    got = analyzer.rvq_encode(channels, books, latent)
    expected = np.zeros((57, books), np.uint16)
    ref_check(ref().ref_rvq_encode(str(package).encode(), channels, books, ptr(latent),
                                   c_size_t(57), ptr(expected)))
    assert np.array_equal(got, expected)
    rec = analyzer.rvq_decode(channels, books, got)
    ref_rec = np.zeros((57, 1024), np.float32)
    ref_check(ref().ref_rvq_decode(str(package).encode(), channels, books, ptr(expected),
                                   c_size_t(57), ptr(ref_rec)))
    assert np.array_equal(rec.view(np.uint32), ref_rec.view(np.uint32))
