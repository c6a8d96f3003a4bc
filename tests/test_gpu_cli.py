"""tsac-cuda end to end on the GPU: `c` writes the reference's golden streams
byte for byte from a WAVE file, `d` writes the decoded PCM as 16-bit WAVE with
the reference's rounding (src/audio.cpp:198-246), `t` round-trips, and `-vv`
prints the statistics lines of src/codec.cpp:41-110."""
from __future__ import annotations

import hashlib
import json
import pathlib
import struct
import subprocess

import numpy as np
import pytest

from support import GOLDEN

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402

ROOT = pathlib.Path(__file__).resolve().parents[1]
CLI = ROOT / "tsac-metal_b200" / "tsac-cuda"


def write_wave(path, pcm):
    ints = np.clip(np.rint(pcm.astype(np.float64) * 32768.0), -32768, 32767).astype("<i2")
    channels = pcm.shape[1]
    data = ints.tobytes()
    header = b"RIFF" + struct.pack("<I", len(data) + 36) + b"WAVE" + b"fmt " + struct.pack(
        "<IHHIIHH", 16, 1, channels, 44100, 44100 * 2 * channels, 2 * channels, 16) + b"data" + \
        struct.pack("<I", len(data))
    path.write_bytes(header + data)


def read_wave(path):
    raw = path.read_bytes()
    assert raw[:4] == b"RIFF" and raw[8:12] == b"WAVE"
    channels = struct.unpack("<H", raw[22:24])[0]
    size = struct.unpack("<I", raw[40:44])[0]
    return channels, np.frombuffer(raw[44:44 + size], "<i2").reshape(-1, channels)


def pcm16(x):
    """The reference's float -> PCM16 rule: scale, clip, round half to even."""
    s = np.clip(np.asarray(x, np.float64) * 32768.0, -32768.0, 32767.0)
    return np.rint(s).astype(np.int16)


def cli(*args):
    r = subprocess.run([str(CLI), "--models", str(tsac_cuda.seeded_package(0)), *args],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return r.stdout


@pytest.mark.parametrize("case", ["stereo_q12_b3_1s", "mono_q9_b2_0p5s", "stereo_fast_q3_0p5s",
                                  "separate_q5_b2_0p5s"])
def test_compress_matches_golden_stream(tmp_path, case):
    g = json.loads((GOLDEN / f"{case}.json").read_text())
    pcm = synthetic.music_like(g["pcm_seed"], g["seconds"], g["channels"])
    write_wave(tmp_path / "in.wav", pcm)
    args = ["-q", str(g["codebooks"]), "-T", "3"]  # a host thread budget changes no byte
    if g["method"] == 0:
        args.append("-f")
    if g["separate"]:
        args.append("-s")
    if g["batch"]:
        args += ["--batch_size", str(g["batch"])]
    cli(*args, "c", str(tmp_path / "in.wav"), str(tmp_path / "out.tsac"))
    stream = (tmp_path / "out.tsac").read_bytes()
    assert hashlib.sha256(stream).hexdigest() == g["stream_sha256"]


def test_decompress_exact_writes_reference_pcm16(tmp_path):
    case = "stereo_q12_b3_1s"
    stream_path = GOLDEN / f"{case}.tsac"
    cli("--exact", "d", str(stream_path), str(tmp_path / "out.wav"))
    channels, got = read_wave(tmp_path / "out.wav")
    analyzer = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    analyzer.set_exact_synthesis(True)
    audio = analyzer.decode(stream_path.read_bytes())
    analyzer.close()
    assert channels == audio.channels
    assert np.array_equal(got.ravel(), pcm16(audio.samples).ravel())


def test_round_trip_and_statistics(tmp_path):
    pcm = synthetic.music_like(77, 0.7, 2)
    write_wave(tmp_path / "in.wav", pcm)
    out = cli("-vv", "-T", "1", "-q", "6", "t", str(tmp_path / "in.wav"), str(tmp_path / "rt.wav"))
    lines = out.splitlines()
    assert lines[0].startswith("batch_size=") and " n_cb=6 " in lines[0]
    assert "CB AVG_BITS" in lines
    table = lines[lines.index("CB AVG_BITS") + 1: lines.index("CB AVG_BITS") + 7]
    assert [int(l.split()[0]) for l in table] == list(range(6))
    assert any(l.startswith("bitrate=") and "kb/s" in l for l in lines)
    channels, got = read_wave(tmp_path / "rt.wav")
    assert channels == 2 and got.shape[0] >= pcm.shape[0] and got.shape[0] % 512 == 0
