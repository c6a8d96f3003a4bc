"""tsac-cuda command line tool: argument handling without a GPU (the
reference's parser rules, src/cli.cpp:6-126) and loud failure when no device
is present."""
from __future__ import annotations

import pathlib
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
CLI = ROOT / "tsac-metal_b200" / "tsac-cuda"


def run(*args):
    if not CLI.exists():
        pytest.skip("tsac-cuda not built")
    return subprocess.run([str(CLI), *args], capture_output=True, text=True, timeout=120)


def test_help_and_usage_exit_1():
    r = run("-h")
    assert r.returncode == 1 and "usage: tsac-cuda" in r.stdout
    r = run()  # fewer than three positionals prints the help too
    assert r.returncode == 1 and "usage: tsac-cuda" in r.stdout


@pytest.mark.parametrize("args,message", [
    (["-q1", "c", "a", "b"], "unknown option: '-1'"),
    (["-x", "c", "a", "b"], "unknown option: '-x'"),
    (["--nope", "c", "a", "b"], "unknown option: '--nope'"),
    (["-q", "abc", "c", "a", "b"], "option --n_codebooks expects an integer"),
    (["-c", "1.5", "c", "a", "b"], "option --channels expects an integer"),
    (["--batch_size"], "option '--batch_size' must have an argument"),
    (["z", "a", "b"], "unknown command: z"),
    (["--metal", "c", "a", "b"], "Metal execution is not available"),
    (["-T", "257", "c", "a", "b"], "CPU thread count exceeds supported limit (256)"),
])
def test_rejected_arguments(args, message):
    r = run(*args)
    assert r.returncode == 1
    assert r.stderr.startswith("tsac-cuda: ") and message in r.stderr


def test_plus_sign_and_grouped_flags_accepted(tmp_path):
    # "+12" parses as 12 and "-vv" counts twice; the run then fails on the
    # missing model package, after parsing succeeded.
    r = run("--models", str(tmp_path), "-vv", "-q", "+12", "c", str(tmp_path / "in.wav"),
            str(tmp_path / "out.tsac"))
    assert r.returncode == 1
    assert "expects an integer" not in r.stderr and "unknown option" not in r.stderr


def _wave(channels=2, rate=44100, bits=16, fmt_tag=1, frames=600, data_size=None, order=("fmt", "data"),
          extra=b""):
    import struct

    import numpy as np
    pcm = (np.arange(frames * channels, dtype=np.int64) * 37 % 65536 - 32768).astype("<i2").tobytes()
    fmt = struct.pack("<HHIIHH", fmt_tag, channels, rate, rate * channels * 2, channels * 2, bits)
    chunks = {"fmt": b"fmt " + struct.pack("<I", len(fmt)) + fmt,
              "data": b"data" + struct.pack("<I", len(pcm) if data_size is None else data_size) + pcm}
    body = b"WAVE" + extra + b"".join(chunks[c] for c in order)
    return b"RIFF" + struct.pack("<I", len(body)) + body


def _no_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")


def test_without_gpu_fails_loudly(tmp_path):
    _no_gpu()
    import tsac_cuda
    (tmp_path / "in.wav").write_bytes(_wave())
    r = run("--models", str(tsac_cuda.seeded_package(0)), "c", str(tmp_path / "in.wav"),
            str(tmp_path / "out.tsac"))
    assert r.returncode == 1 and "no CUDA device" in r.stderr


@pytest.mark.parametrize("kwargs,message", [
    (dict(rate=48000), "the sample rate must be 44100 Hz"),
    (dict(channels=9), "unsupported number of channels"),
    (dict(bits=24), "invalid wav file"),
    (dict(fmt_tag=3), "invalid wav file"),
    (dict(order=("data", "fmt")), "invalid wav file"),
    (dict(order=("fmt",)), "invalid wav file"),
])
def test_wave_input_rejections(tmp_path, kwargs, message):
    """The native WAVE reader's checks (wave_input, src/audio.cpp:39-73) run
    before any device work."""
    (tmp_path / "in.wav").write_bytes(_wave(**kwargs))
    r = run("--models", str(tmp_path), "c", str(tmp_path / "in.wav"), str(tmp_path / "out.tsac"))
    assert r.returncode == 1 and message in r.stderr, r.stderr


@pytest.mark.parametrize("kwargs", [dict(data_size=0xFFFFFFF0), dict(extra=b"LIST\x04\x00\x00\x00abcd"),
                                    dict(channels=8, frames=3)])
def test_wave_input_accepted(tmp_path, kwargs):
    """A data chunk is read to the end of the file whatever size it declares,
    unknown chunks are skipped: parsing succeeds and the run stops only at the
    missing device."""
    _no_gpu()
    import tsac_cuda
    (tmp_path / "in.wav").write_bytes(_wave(**kwargs))
    r = run("--models", str(tsac_cuda.seeded_package(0)), "c", str(tmp_path / "in.wav"),
            str(tmp_path / "out.tsac"))
    assert r.returncode == 1 and "no CUDA device" in r.stderr, r.stderr


def test_truncated_riff_rejected(tmp_path):
    data = _wave()
    for size in (0, 4, 11, 12 + 6):
        (tmp_path / "in.wav").write_bytes(data[:size])
        r = run("--models", str(tmp_path), "c", str(tmp_path / "in.wav"), str(tmp_path / "out.tsac"))
        assert r.returncode == 1 and "invalid wav file" in r.stderr, (size, r.stderr)
