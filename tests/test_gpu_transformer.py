"""GPU probability model vs the reference: byte-identical normal-mode streams.

The known-token header shapes are those of the reference's own GPU-vs-CPU
known-token test (tests/metal_optimized.cpp:252-270): (frames, batch, groups),
joint stereo, 12 books (1 book for the 1026-frame case, which crosses the
1024-position context and exercises the 256-frame replay).  Expected streams and
per-symbol probability-row CRCs were produced by the reference scalar path
(tests/golden/make_golden.py --cases known).
"""
import binascii
import hashlib
import json

import numpy as np
import pytest

from support import GOLDEN, c_size_t, ptr, ref, ref_available, ref_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402

KNOWN = sorted(p.stem for p in GOLDEN.glob("known_*.json"))


@pytest.fixture(scope="module")
def analyzer():
    a = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    yield a
    a.close()


def _tokens(frames, groups, books):
    i = np.arange(frames * groups * books, dtype=np.int64)
    return ((i * 73 + 19) % 1024).astype(np.uint16)


@pytest.mark.parametrize("case", KNOWN)
def test_known_token_stream_matches_reference(analyzer, case):
    g = json.loads((GOLDEN / f"{case}.json").read_text())
    tokens = _tokens(g["frames"], g["groups"], g["books"])
    stream = analyzer.pack_normal(g["channels"], g["groups"], g["books"], g["frames"], g["batch"],
                                  tokens)
    if hashlib.sha256(stream).hexdigest() != g["stream_sha256"]:
        probs, _ = analyzer.transformer_probabilities(g["channels"], g["groups"], g["books"],
                                                      g["frames"], g["batch"], tokens)
        crc = [binascii.crc32(row.tobytes()) for row in probs]
        bad = [i for i, (a, b) in enumerate(zip(crc, g["probability_row_crc32"])) if a != b]
        pytest.fail(f"stream differs ({len(stream)} vs {g['stream_bytes']} bytes); "
                    f"{len(bad)} probability rows differ, first {bad[:8]}")


def test_probabilities_match_live_reference(analyzer):
    if not ref_available():
        pytest.skip("reference oracle not built")
    package = tsac_cuda.seeded_package(0)
    frames, batch, groups, books = 5, 2, 2, 12
    tokens = _tokens(frames, groups, books)
    probs, q15 = analyzer.transformer_probabilities(2, groups, books, frames, batch, tokens)
    expected = np.zeros_like(probs)
    ref_check(ref().ref_transformer_probabilities(str(package).encode(), 2, groups, books,
                                                  c_size_t(frames), batch, ptr(tokens),
                                                  ptr(expected)))
    # The reference writes rows in entropy order; ours are in token-offset order.
    order = []
    per_lane, extra = frames // batch, frames % batch
    for step in range(per_lane + (extra != 0)):
        for book in range(books):
            for lane in range(min(batch, frames)):
                if step >= per_lane + (lane < extra):
                    continue
                frame = lane * per_lane + min(lane, extra) + step
                for g in range(groups):
                    order.append((frame * groups + g) * books + book)
    assert np.array_equal(probs[order].view(np.uint32), expected.view(np.uint32))
