"""Whole-codec parity: CudaAnalyzer vs the reference ScalarAnalyzer.

Golden streams/PCM hashes come from the reference scalar path on the seeded
package (tests/golden/make_golden.py).  Streams must be byte-identical.
Decoded PCM: with exact synthesis (the serial kernels keep the reference's
operation order) it is compared bit for bit; with the default tensor-core
synthesis it must agree with the exact PCM within the reference's own pipeline
tolerance |a - b| <= 1e-4 * (1 + max(|a|, |b|)) (tests/metal_optimized.cpp:741-745
of the reference).  Every stream must decode on either side.  The failure cases
follow tests/audio_analyzer.cpp:307-425 of the reference.
"""
import hashlib
import json
import pathlib

import numpy as np
import pytest

from support import GOLDEN

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402

CASES = sorted(p.stem for p in GOLDEN.glob("*.json")
               if not p.stem.startswith("known_") and p.stem not in ("cfg0_stereo_30s", "cfg3_mono_60s"))


PCM_RTOL = 1e-4  # |a - b| <= PCM_RTOL * (1 + max(|a|, |b|))


@pytest.fixture(scope="module")
def analyzer():
    a = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    yield a
    a.close()


@pytest.fixture(scope="module")
def exact_analyzer():
    a = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    a.set_exact_synthesis(True)
    yield a
    a.close()


def assert_pcm_close(got, expected):
    got, expected = np.asarray(got, np.float64), np.asarray(expected, np.float64)
    assert got.shape == expected.shape
    bound = PCM_RTOL * (1.0 + np.maximum(np.abs(got), np.abs(expected)))
    excess = np.abs(got - expected) - bound
    assert excess.max() <= 0, (f"{int((excess > 0).sum())} of {got.size} samples outside tolerance; "
                               f"max |d| {np.abs(got - expected).max():.3g}")


def _golden(case):
    return json.loads((GOLDEN / f"{case}.json").read_text())


def _options(g):
    return tsac_cuda.EncodeOptions(method="normal" if g["method"] == 1 else "fast",
                                   codebooks=g["codebooks"], separate_channels=bool(g["separate"]),
                                   entropy_batch=g["batch"] or None)


@pytest.mark.parametrize("case", CASES)
def test_encode_stream_byte_identical(analyzer, case):
    g = _golden(case)
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    stream = analyzer.encode(pcm, _options(g))
    assert len(stream) == g["stream_bytes"]
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]


@pytest.mark.parametrize("case", CASES)
def test_decode_reference_stream_bit_exact(exact_analyzer, case):
    g = _golden(case)
    stream = (GOLDEN / f"{case}.tsac").read_bytes()
    audio = exact_analyzer.decode(stream)
    assert audio.channels == g["pcm_channels"] and audio.samples.size == g["pcm_samples"]
    head = np.array(g["pcm_head"], np.float32)
    flat = audio.samples.ravel()
    assert np.array_equal(flat[: head.size].view(np.uint32), head.view(np.uint32)), \
        f"max |d| {np.abs(flat[:head.size] - head).max()}"
    assert hashlib.sha256(flat.astype("<f4").tobytes()).hexdigest() == g["pcm_sha256"]


def test_cfg0_full_clip_stream_and_pcm(analyzer, exact_analyzer):
    """cfg0: 30 s joint stereo, seed 0, q=12, batch 3 (2,584 frames, lanes
    862/861/861): the stream is byte-identical to the reference's, and exact
    decoding reproduces the reference's PCM bit for bit."""
    g = _golden("cfg0_stereo_30s")
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    stream = analyzer.encode(pcm, _options(g))
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]
    audio = exact_analyzer.decode(stream)
    flat = audio.samples.ravel()
    assert hashlib.sha256(flat.astype("<f4").tobytes()).hexdigest() == g["pcm_sha256"]
    fast = analyzer.decode(stream)
    assert_pcm_close(fast.samples, audio.samples)


@pytest.mark.parametrize("case", CASES)
def test_decode_tensor_synthesis_within_tolerance(analyzer, exact_analyzer, case):
    stream = (GOLDEN / f"{case}.tsac").read_bytes()
    got = analyzer.decode(stream)
    expected = exact_analyzer.decode(stream)
    assert got.channels == expected.channels
    assert_pcm_close(got.samples, expected.samples)


def test_decode_batch_tensor_synthesis_within_tolerance(analyzer, exact_analyzer):
    # Several recordings of different lengths, one longer than a synthesis
    # chunk (400 frames), decoded as one batch: every window becomes a
    # sequence of the padded layout, so edges and gaps are exercised.
    opts = tsac_cuda.EncodeOptions(method="normal", codebooks=3, entropy_batch=4)
    pcms = [synthetic.music_like(900 + i, s, 2) for i, s in enumerate((0.05, 5.2, 1.3, 0.6))]
    streams = exact_analyzer.encode_batch(pcms, opts)
    got = analyzer.decode_batch(streams)
    expected = exact_analyzer.decode_batch(streams)
    for g_, e_ in zip(got, expected):
        assert_pcm_close(g_.samples, e_.samples)


def test_batch_equals_single(analyzer):
    cases = [c for c in CASES if _golden(c)["seconds"] >= 0.05][:4]
    pcms = [synthetic.music_like(_golden(c)["pcm_seed"], _golden(c)["seconds"], _golden(c)["channels"])
            for c in cases]
    opts = tsac_cuda.EncodeOptions()
    single = [analyzer.encode(p, opts) for p in pcms]
    assert analyzer.encode_batch(pcms, opts) == single
    decoded = analyzer.decode_batch(single)
    for s, d in zip(single, decoded):
        one = analyzer.decode(s)
        assert np.array_equal(one.samples, d.samples)


def test_strided_views_give_identical_streams(analyzer):
    pcm = synthetic.music_like(31, 0.2, 2)
    planar = np.ascontiguousarray(pcm.T).T  # channel-major memory, same values
    assert analyzer.encode(pcm) == analyzer.encode(planar)


def test_failures_are_errors_and_analyzer_is_reusable(analyzer):
    pcm = synthetic.music_like(32, 0.05, 2)
    bad = pcm.copy()
    bad[10, 1] = np.nan
    with pytest.raises(tsac_cuda.TsacError, match="nonfinite PCM"):
        analyzer.encode(bad)
    with pytest.raises(tsac_cuda.TsacError, match="codebooks"):
        analyzer.encode(pcm, tsac_cuda.EncodeOptions(codebooks=13))
    with pytest.raises(tsac_cuda.TsacError, match="normal coding"):
        analyzer.encode(pcm, tsac_cuda.EncodeOptions(method="fast", entropy_batch=2))
    with pytest.raises(tsac_cuda.TsacError):
        analyzer.decode(b"")
    stream = bytearray(analyzer.encode(pcm))
    stream[-1] ^= 1  # corrupt the token CRC
    with pytest.raises(tsac_cuda.TsacError, match="CRC"):
        analyzer.decode(bytes(stream))
    # Reuse after failures.
    good = analyzer.encode(pcm)
    assert analyzer.decode(good).samples.shape == (512 * 5, 2)


def _entropy_books(frames, batch, groups, books):
    """Codebook of each symbol in visit_entropy_positions order (step, book,
    lane, group; src/format/entropy.cpp:26-55)."""
    lanes = min(batch, frames)
    base, extra = divmod(frames, batch)
    length = [base + (lane < extra) for lane in range(lanes)]
    order = []
    for step in range(max(length)):
        for book in range(books):
            for lane in range(lanes):
                if step < length[lane]:
                    order += [book] * groups
    return np.array(order)


@pytest.mark.parametrize("case", ["stereo_q12_b3_1s", "separate_q5_b2_0p5s", "stereo_fast_q3_0p5s"])
def test_symbol_bits_for_observers(analyzer, case):
    """Each symbol's bits in entropy order, what an EntropyObserver's
    after_symbol receives: one per symbol, summing to the reference's payload
    bit count and, per codebook, to the observed per-codebook totals; fast
    streams have none."""
    import ctypes

    g = _golden(case)
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    stream, per_symbol = analyzer.encode_symbol_bits(pcm, _options(g))
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]
    if g["method"] == 0:
        assert per_symbol.size == 0
        return
    assert per_symbol.size == g["tokens"]
    assert int(per_symbol.sum(dtype=np.int64)) == g["symbol_bits"]
    channels, _, _ = tsac_cuda.stream_info(stream)
    groups = channels if (g["separate"] or channels == 1) else 1
    frames = (int(pcm.shape[0]) + 511) // 512
    books = _entropy_books(frames, g["batch"], groups, g["codebooks"])
    totals = (ctypes.c_uint64 * g["codebooks"])()
    out, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
    pcm32 = np.ascontiguousarray(pcm, dtype=np.float32)
    opts = tsac_cuda._options(_options(g))
    tsac_cuda.check(tsac_cuda.library().tsac_cuda_encode_observed(
        analyzer._ctx, pcm32.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(pcm32.shape[1]),
        ctypes.c_size_t(pcm32.shape[0]), ctypes.c_ssize_t(1), ctypes.c_ssize_t(pcm32.shape[1]),
        ctypes.byref(opts), ctypes.byref(out), ctypes.byref(nbytes), totals, ctypes.c_size_t(g["codebooks"])))
    tsac_cuda.library().tsac_cuda_free(out)
    expected = np.bincount(books, weights=per_symbol, minlength=g["codebooks"]).astype(np.int64)
    assert list(expected) == list(totals)


def test_host_thread_budget(analyzer):
    """Range coding under a host thread budget (the reference CLI's -T, 1-256)
    gives the same streams and the same decoded PCM; larger budgets are errors."""
    pcms = [synthetic.music_like(40 + i, 0.3, 2) for i in range(3)]
    automatic = analyzer.encode_batch(pcms)
    reference = analyzer.decode_batch(automatic)
    try:
        for threads in (1, 2, 3):
            analyzer.set_host_threads(threads)
            assert analyzer.encode_batch(pcms) == automatic
            for got, want in zip(analyzer.decode_batch(automatic), reference):
                assert np.array_equal(got.samples, want.samples)
        with pytest.raises(tsac_cuda.TsacError, match="256"):
            analyzer.set_host_threads(257)
    finally:
        analyzer.set_host_threads(0)


@pytest.mark.parametrize("case", ["known_17_8_16", "known_101_3_1", "known_35_3_2", "known_17_1_1",
                                  "known_3_8_2", "known_1026_1_1", "known_mono_40_2_1"])
def test_decode_known_token_streams(analyzer, case):
    """The reference's own streams of known tokens decode on the GPU-resident
    loop: 16 channel groups, batches 1..8, mono, and 1026 frames at batch 1,
    which replays the last 256 frames after 1024 (a different row shape for
    that step).  The decoder checks the stream's token CRC-32, so a wrong
    token anywhere fails the call."""
    g = _golden(case)
    stream = (GOLDEN / f"{case}.tsac").read_bytes()
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]
    decoded = analyzer.decode(stream)
    assert decoded.samples.shape == (g["frames"] * 512, g["channels"] * g["groups"])


def test_decode_batch_mixed_shapes_equals_single(analyzer):
    """One decode batch holding recordings of different lengths, codebook
    counts, channel groups and entropy batches (lanes end at different steps
    and books, so the loop runs several row shapes) decodes each exactly as
    alone."""
    names = ["stereo_q12_b3_1s", "separate_q5_b2_0p5s", "stereo_q1_b7_0p3s", "stereo_q4_b8_0p05s",
             "known_35_3_2", "stereo_q12_auto_0p1s"]
    streams = [(GOLDEN / f"{n}.tsac").read_bytes() for n in names]
    singles = [analyzer.decode(s).samples for s in streams]
    for got, want in zip(analyzer.decode_batch(streams), singles):
        assert np.array_equal(got.samples.view(np.uint32), want.view(np.uint32))


def test_corrupt_payload_is_an_error_and_analyzer_is_reusable(analyzer):
    """Flipped payload bytes make the device range decoder leave its interval
    or decode wrong tokens: the call fails (range error or token CRC) and the
    next call on the same analyzer succeeds."""
    stream = bytearray((GOLDEN / "stereo_q12_b3_1s.tsac").read_bytes())
    for at in (14, 15, 40, len(stream) // 2):
        bad = bytearray(stream)
        bad[at] ^= 0xFF
        with pytest.raises(tsac_cuda.TsacError, match="range code|CRC"):
            analyzer.decode(bytes(bad))
    truncated = bytes(stream[:40]) + bytes(stream[-4:])
    with pytest.raises(tsac_cuda.TsacError):
        analyzer.decode(truncated)
    assert analyzer.decode(bytes(stream)).samples.shape[1] == 2
