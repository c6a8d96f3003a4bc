"""The certified fast analysis (tsac_cuda_set_fast_analysis): fused
multiply-add analysis convolutions, every RVQ decision's lead over its
runner-up checked against a margin, and frames below it recomputed exactly on
their 17-frame sub-windows.  Streams must stay byte-identical to the
reference's goldens at any margin:
  - margin 2 (every similarity lies in [-1, 1], so every frame is flagged):
    the whole encoder runs through the sub-window recomputation, which checks
    that a frame's exact latent depends only on its +-8-frame reach;
  - a working margin (1e-4): most frames keep their fast tokens.
The counters report how many frames were flagged and recomputed."""
import hashlib
import json

import numpy as np
import pytest

from support import GOLDEN

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402

CASES = ["stereo_q12_b3_1s", "mono_q9_b2_0p5s", "separate_q5_b2_0p5s", "stereo_q12_auto_0p1s",
         "stereo_q1_b7_0p3s", "stereo_q4_b8_0p05s", "stereo_fast_q3_0p5s", "mono_q2_one_sample"]


@pytest.fixture(scope="module")
def analyzer():
    a = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    yield a
    a.close()


def _encode(a, case):
    g = json.loads((GOLDEN / f"{case}.json").read_text())
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    o = tsac_cuda.EncodeOptions(method="normal" if g["method"] == 1 else "fast", codebooks=g["codebooks"],
                                separate_channels=bool(g["separate"]), entropy_batch=g["batch"] or None)
    return hashlib.sha256(a.encode(pcm, o)).hexdigest() == g["stream_sha256"]


@pytest.mark.parametrize("margin", [2.0, 1e-4])
def test_fast_analysis_streams_byte_identical(analyzer, margin):
    analyzer.set_fast_analysis(margin)
    try:
        before = analyzer.fast_analysis_stats()
        assert all(_encode(analyzer, c) for c in CASES)
        frames, flagged, recomputed = (x - y for x, y in zip(analyzer.fast_analysis_stats(), before))
        assert frames > 0
        if margin == 2.0:
            assert flagged == frames and recomputed >= frames
        else:
            assert flagged < frames
    finally:
        analyzer.set_fast_analysis(0.0)


def test_fast_analysis_cfg0_clip_byte_identical(analyzer):
    """The 30 s cfg0 clip (2,584 frames, 7 analysis windows) at the working margin."""
    g = json.loads((GOLDEN / "cfg0_stereo_30s.json").read_text())
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    analyzer.set_fast_analysis(1e-4)
    try:
        stream = analyzer.encode(pcm, tsac_cuda.EncodeOptions(method="normal", codebooks=12, entropy_batch=3))
    finally:
        analyzer.set_fast_analysis(0.0)
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]


def test_fast_latents_close_to_exact(analyzer):
    """The fused path's latents stay within 1e-4 of the exact ones relative to
    each frame's RMS (measured about 1.7e-5 at most)."""
    pcm = synthetic.music_like(3, 2.0, 2)
    pcm = pcm[: (pcm.shape[0] // 512) * 512]
    exact = analyzer.dac_analysis(2, pcm)
    analyzer.set_fast_analysis(1e-4)
    try:
        fast = analyzer.dac_analysis(2, pcm)
    finally:
        analyzer.set_fast_analysis(0.0)
    rms = np.sqrt((exact.astype(np.float64) ** 2).mean(axis=1, keepdims=True))
    rel = np.abs(fast.astype(np.float64) - exact) / rms
    assert rel.max() < 1e-4
    assert not np.array_equal(fast, exact)  # it is a different arithmetic


def test_margin_out_of_range_rejected(analyzer):
    with pytest.raises(tsac_cuda.TsacError, match="margin"):
        analyzer.set_fast_analysis(-1.0)
