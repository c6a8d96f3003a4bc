"""cfg3, DAC-only decode: 60 s of mono at 9 codebooks (5,168 frames), tokens
uniform in [0, 1024) from seed 3, packed as a fast (method 0) stream, decoded
to PCM by the reference scalar path (tests/golden/make_golden.py, the golden
cfg3_mono_60s.{json,tsac}; src/common/synthesis.tpp:168-213 and
src/common/audio_pipeline.hpp:63-83 of the reference).

Exact synthesis must reproduce the reference's PCM bit for bit (sha256 of the
whole 60 s); the default tensor-core synthesis must stay within the
reference's pipeline tolerance |a - b| <= 1e-4 (1 + max(|a|, |b|)) of it."""
import hashlib
import json

import numpy as np
import pytest

from support import GOLDEN

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402

CASE = GOLDEN / "cfg3_mono_60s.json"


@pytest.fixture(scope="module")
def decoded():
    if not CASE.exists():
        pytest.skip("cfg3 golden not generated")
    g = json.loads(CASE.read_text())
    stream = (GOLDEN / "cfg3_mono_60s.tsac").read_bytes()
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]
    a = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    a.set_exact_synthesis(True)
    exact = a.decode(stream)
    a.set_exact_synthesis(False)
    tensor = a.decode(stream)
    a.close()
    return g, exact, tensor


def test_cfg3_stream_shape(decoded):
    g, exact, _ = decoded
    assert exact.channels == 1 and g["frames"] == 5168 and g["books"] == 9
    assert exact.samples.size == g["pcm_samples"] == 5168 * 512


def test_cfg3_exact_pcm_bit_identical(decoded):
    g, exact, _ = decoded
    flat = exact.samples.ravel().astype("<f4")
    assert np.array_equal(flat[:4096], np.asarray(g["pcm_head"], np.float32))
    assert hashlib.sha256(flat.tobytes()).hexdigest() == g["pcm_sha256"]


def test_cfg3_tensor_pcm_within_tolerance(decoded):
    _, exact, tensor = decoded
    a = exact.samples.astype(np.float64).ravel()
    b = tensor.samples.astype(np.float64).ravel()
    bound = 1e-4 * (1.0 + np.maximum(np.abs(a), np.abs(b)))
    excess = np.abs(a - b) - bound
    assert excess.max() <= 0, f"{int((excess > 0).sum())} samples outside; max |d| {np.abs(a - b).max():.3g}"
