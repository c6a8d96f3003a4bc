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


def test_without_gpu_fails_loudly(tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import tsac_cuda
    r = run("--models", str(tsac_cuda.seeded_package(0)), "c", str(tmp_path / "in.wav"),
            str(tmp_path / "out.tsac"))
    assert r.returncode == 1 and "no CUDA device" in r.stderr
