"""Container and packaging checks that need no GPU.

Container known answers follow the reference's sanitation test
(tests/sanitation.cpp:34-105): the 11-byte fast stream decodes to tokens
[987, 90], every truncation but the bare 8-byte header is rejected, the listed
single-byte corruptions are rejected, and the 19-byte normal header carries
the token CRC 0x895ce095 of those tokens.  The packer check compares this
library's packer with the reference packer (oracle/_ref/tsac-pack-models, built
from the reference sources) byte for byte on the same seeded originals.
"""
from __future__ import annotations

import filecmp
import pathlib
import subprocess

import numpy as np
import pytest

import tsac_cuda

ROOT = pathlib.Path(__file__).resolve().parents[1]
REF_PACKER = ROOT / "oracle" / "_ref" / "tsac-pack-models"

FAST = bytes([ord("F"), ord("B"), ord("A"), ord("Z"), 0, 0, 1, 1, 0xF6, 0xC5, 0xA0])
NORMAL = bytes([ord("F"), ord("B"), ord("A"), ord("Z"), 0, 1, 1, 1, 0, 0, 0, 2, 0, 1, 0,
                0x89, 0x5C, 0xE0, 0x95])


def rejects(fn, *args):
    with pytest.raises(tsac_cuda.TsacError):
        fn(*args)


def test_fast_stream_known_answer():
    assert tsac_cuda.unpack_fast(FAST).tolist() == [987, 90]
    channels, samples, symbols = tsac_cuda.stream_info(FAST)
    assert (channels, symbols) == (1, 2)
    assert samples > 0


def test_fast_stream_truncations_rejected():
    for size in range(len(FAST)):
        if size == 8:
            tsac_cuda.stream_info(FAST[:size])  # a bare header parses
            continue
        rejects(tsac_cuda.stream_info, FAST[:size])


@pytest.mark.parametrize("offset,value", [(0, 0), (4, 1), (5, 2), (6, 0), (7, 0), (7, 10),
                                          (10, 0xA1)])
def test_fast_stream_corruptions_rejected(offset, value):
    bad = bytearray(FAST)
    bad[offset] = value
    rejects(tsac_cuda.stream_info, bytes(bad))


def test_normal_header_token_crc():
    assert tsac_cuda.token_crc32(np.array([987, 90], np.uint16)) == 0x895CE095
    assert tsac_cuda.stream_info(NORMAL)[2] == 2
    for size in range(len(NORMAL)):
        rejects(tsac_cuda.stream_info, NORMAL[:size])
    bad = bytearray(NORMAL)
    bad[13] = 0
    rejects(tsac_cuda.stream_info, bytes(bad))


def test_token_crc_changes_with_every_token():
    tokens = np.arange(64, dtype=np.uint16) * 7 % 1024
    base = tsac_cuda.token_crc32(tokens)
    for i in range(0, 64, 9):
        t = tokens.copy()
        t[i] ^= 1
        assert tsac_cuda.token_crc32(t) != base


def _crc32_msb_first(tokens):
    """The token CRC restated bit by bit: polynomial 0x04c11db7, MSB first,
    initial ~0, no final xor, over each token's four little-endian bytes."""
    reg = 0xFFFFFFFF
    for t in tokens.tolist():
        for byte in int(t).to_bytes(4, "little"):
            reg ^= byte << 24
            for _ in range(8):
                reg = ((reg << 1) ^ 0x04C11DB7 if reg & 0x80000000 else reg << 1) & 0xFFFFFFFF
    return reg


@pytest.mark.parametrize("count", [0, 1, 3, 257, 1000])
def test_token_crc_matches_bitwise_definition(count):
    tokens = np.random.default_rng(count).integers(0, 1024, count).astype(np.uint16)
    assert tsac_cuda.token_crc32(tokens) == _crc32_msb_first(tokens)


@pytest.mark.parametrize("groups,books,frames", [(1, 1, 1), (1, 9, 7), (2, 12, 3), (3, 5, 11),
                                                 (1, 12, 64), (5, 3, 2)])
def test_fast_unpack_of_reference_packed_streams(groups, books, frames):
    """Streams packed by the reference's pack_fast (every token count modulo
    4, so every tail of the 40-bit words) unpack to the same tokens."""
    import ctypes

    from support import ptr, ref, ref_check

    channels = 2 if books > 9 else 1
    tokens = np.random.default_rng(groups * 100 + books * 10 + frames).integers(
        0, 1024, frames * groups * books).astype(np.uint16)
    out, size = ctypes.POINTER(ctypes.c_uint8)(), ctypes.c_size_t()
    ref_check(ref().ref_pack_fast(channels, groups, books, ctypes.c_size_t(frames), ptr(tokens),
                                  ctypes.byref(out), ctypes.byref(size)))
    stream = bytes(out[: size.value])
    ref().ref_free(out)
    assert np.array_equal(tsac_cuda.unpack_fast(stream), tokens)
    assert tsac_cuda.stream_info(stream)[2] == tokens.size


@pytest.mark.slow
def test_packer_matches_reference_packer(tmp_path):
    if not REF_PACKER.exists():
        pytest.skip("reference packer oracle/_ref/tsac-pack-models not built")
    source = tmp_path / "source"
    ours, theirs = tmp_path / "ours", tmp_path / "theirs"
    tsac_cuda.write_seeded_sources(source, 3)
    tsac_cuda.pack_models(source, ours, "0123456789abcdef", include_transformer=True)
    subprocess.run([str(REF_PACKER), str(source), str(theirs), "0123456789abcdef", "1"],
                   check=True, capture_output=True)
    ours_files = sorted(p.name for p in ours.iterdir())
    theirs_files = sorted(p.name for p in theirs.iterdir())
    assert ours_files == theirs_files
    assert len(ours_files) == 20 + 2  # 20 weight files, adapter header, manifest
    for name in ours_files:
        assert filecmp.cmp(ours / name, theirs / name, shallow=False), name
    total = sum((ours / n).stat().st_size for n in ours_files if n.endswith(".weights"))
    assert total == 317_259_776


def _generate_package(args):
    cache, seed = args
    import os

    os.environ["TSAC_B200_CACHE"] = cache
    import tsac_cuda

    return str(tsac_cuda.seeded_package(seed))


@pytest.mark.slow
def test_seeded_package_concurrent_generation(tmp_path):
    """One process per GPU on a fresh host may ask for the seeded package at
    once: one generates it, the others wait and reuse it, and no partial
    directory is left behind."""
    import multiprocessing

    with multiprocessing.get_context("spawn").Pool(4) as pool:
        paths = pool.map(_generate_package, [(str(tmp_path), 3)] * 4)
    package = tmp_path / "seed3" / "package"
    assert set(paths) == {str(package)}
    assert (package / "weights-manifest.cmake").exists()
    assert len(list(package.glob("*.weights"))) == 20
    assert not list((tmp_path / "seed3").glob("package.tmp*"))
