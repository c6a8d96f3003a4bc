"""Seeded synthetic inputs standing in for the reference benchmark's unnamed
"30 seconds of music" (README.md:43-46 of the reference).

cfg0 audio: 8 sines with log-uniform frequencies in [40 Hz, 16 kHz], an
independent uniform phase per channel and equal amplitudes, plus pink noise
(Voss-McCartney, 16 rows), normalised to a -12 dBFS peak (0.2512) and quantised
to PCM16 with round-half-even, then returned as normalised float32 exactly as a
PCM16 WAVE reader would (sample / 32768, src/audio.cpp:19-37).

cfg3 tokens: codes uniform in [0, 1024) for every (frame, book).
"""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 44100
HOP = 512


def pink_noise(rng: np.random.Generator, samples: int, rows: int = 16) -> np.ndarray:
    """Voss-McCartney pink noise: row k holds a uniform value redrawn every 2**k samples."""
    total = np.zeros(samples, dtype=np.float64)
    for k in range(rows):
        period = 1 << k
        draws = rng.uniform(-1.0, 1.0, size=(samples + period - 1) // period)
        total += np.repeat(draws, period)[:samples]
    total += rng.uniform(-1.0, 1.0, size=samples)  # white row
    return total / (rows + 1)


def music_like(seed: int, seconds: float, channels: int = 2) -> np.ndarray:
    """Interleaved float32 PCM [samples][channels] on the PCM16 grid."""
    rng = np.random.default_rng(seed)
    samples = int(round(seconds * SAMPLE_RATE))
    t = np.arange(samples, dtype=np.float64) / SAMPLE_RATE
    x = np.zeros((samples, channels), dtype=np.float64)
    freqs = np.exp(rng.uniform(np.log(40.0), np.log(16000.0), size=8))
    for f in freqs:
        for c in range(channels):
            x[:, c] += np.sin(2.0 * np.pi * f * t + rng.uniform(0.0, 2.0 * np.pi))
    tone_rms = float(np.sqrt(np.mean(x**2))) if samples else 1.0
    for c in range(channels):
        noise = pink_noise(rng, samples)
        noise_rms = float(np.sqrt(np.mean(noise**2))) if samples else 1.0
        x[:, c] += noise * (0.5 * tone_rms / max(noise_rms, 1e-12))
    peak = float(np.abs(x).max()) if samples else 1.0
    x *= 0.2512 / max(peak, 1e-12)
    pcm16 = np.clip(np.rint(x * 32768.0), -32768, 32767)  # rint: half-even
    return (pcm16 / 32768.0).astype(np.float32)


def uniform_tokens(seed: int, frames: int, groups: int, books: int) -> np.ndarray:
    """Tokens [frames][groups][books] uniform in [0, 1024)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 1024, size=(frames, groups, books), dtype=np.uint16)
