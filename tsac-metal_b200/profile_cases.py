#!/usr/bin/env python3
"""Small, deterministic GPU workloads for profiling the library's kernels.

Each case runs one kernel family on a case small enough for an `ncu` capture
(a few seconds of audio, inputs still larger than L2 where it matters) and
exits 0; the NVTX range "case" brackets the measured call, so a capture can
select it with `--nvtx --nvtx-include case/`.

    python tsac-metal_b200/profile_cases.py analysis  [seconds]   # exact DAC encoder
    python tsac-metal_b200/profile_cases.py synthesis [frames]    # tensor-core DAC decoder
    python tsac-metal_b200/profile_cases.py decode    [clips]     # Transformer decode steps

Weights: the seeded package (seed 0); PCM: synthetic.music_like.
"""
from __future__ import annotations

import pathlib
import sys

import numpy as np

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))

import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402


def _range(torch, name):
    class _R:
        def __enter__(self):
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push(name)

        def __exit__(self, *exc):
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    return _R()


def main() -> int:
    import torch

    case = sys.argv[1] if len(sys.argv) > 1 else "synthesis"
    arg = sys.argv[2] if len(sys.argv) > 2 else None
    analyzer = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), 0)
    if case == "analysis":
        seconds = float(arg or 4.0)
        pcm = synthetic.music_like(3, seconds, 2)
        pcm = pcm[: (pcm.shape[0] // 512) * 512]
        analyzer.dac_analysis(2, pcm)  # warm
        with _range(torch, "case"):
            latent = analyzer.dac_analysis(2, pcm)
        print("analysis", latent.shape)
    elif case == "synthesis":
        frames = int(arg or 172)
        tokens = np.random.default_rng(1).integers(0, 1024, (frames, 12)).astype(np.uint16)
        latent = analyzer.rvq_decode(2, 12, tokens)
        analyzer.dac_synthesis(2, latent)  # warm
        with _range(torch, "case"):
            pcm = analyzer.dac_synthesis(2, latent)
        print("synthesis", pcm.shape)
    elif case == "decode":
        clips = int(arg or 16)
        opts = tsac_cuda.EncodeOptions(method="normal", codebooks=12, entropy_batch=3)
        pcms = [synthetic.music_like(i, 0.05, 2) for i in range(clips)]
        streams = analyzer.encode_batch(pcms, opts)
        analyzer.decode_batch(streams)  # warm (captures the step graphs)
        with _range(torch, "case"):
            decoded = analyzer.decode_batch(streams)
        print("decode", len(decoded))
    else:
        print(f"unknown case {case!r}", file=sys.stderr)
        return 2
    analyzer.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
