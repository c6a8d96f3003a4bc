"""The C++ drop-in, tsac::CudaAnalyzer (tsac-metal_b200/adapter), on the GPU
through the reference's own AudioAnalyzer interface: the contract binary runs
the reference's analyzer contract cases (tests/audio_analyzer.cpp:148-425 of
the reference) on it and must report success.

The binary is built where the reference sources are (__graft_entry__.build()
with TSAC_REFERENCE set, or the adapter Makefile) and travels with the tree."""
import pathlib
import subprocess

import pytest

pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402

BINARY = pathlib.Path(__file__).resolve().parents[1] / "tsac-metal_b200" / "adapter" / "_build" / \
    "cuda_analyzer_contract"


def test_cuda_analyzer_keeps_the_reference_contract():
    if not BINARY.exists():
        pytest.skip("adapter contract binary not built (needs the reference sources)")
    r = subprocess.run([str(BINARY), str(tsac_cuda.seeded_package(0))], capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("contract: ok"), r.stdout
