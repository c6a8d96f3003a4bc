"""Generate golden fixtures by running the REFERENCE scalar path (oracle/_ref).

Each case writes tests/golden/<case>.json (hashes, sizes, settings) and, for
small streams, tests/golden/<case>.tsac.  Weights come from the seeded package
(tsac_cuda.seeded_package(0): seeded libnc originals packed into the 20-file
package); PCM comes from synthetic.music_like.  Run here, where the reference
sources exist; the fixtures then travel with the repository.

    python tests/golden/make_golden.py --cases short
    python tests/golden/make_golden.py --cases cfg0_stereo_30s
    python tests/golden/make_golden.py --cases known
    python tests/golden/make_golden.py --cases cfg4 --jobs 6
    python tests/golden/make_golden.py --cases cfg3_mono_60s
"""
from __future__ import annotations

import argparse
import concurrent.futures
import ctypes
import multiprocessing
import hashlib
import json
import pathlib
import sys
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "tsac-metal_b200"))
import synthetic  # noqa: E402
import tsac_cuda  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
REF = ROOT / "oracle" / "_ref" / "libtsac_ref.so"

# name: (pcm seed, seconds, channels, method, codebooks, separate, batch)
CASES = {
    "stereo_q12_auto_0p1s": (1, 0.1, 2, 1, 0, 0, 0),
    "stereo_q12_b3_1s": (2, 1.0, 2, 1, 12, 0, 3),
    "mono_q9_b2_0p5s": (3, 0.5, 1, 1, 0, 0, 2),
    "separate_q5_b2_0p5s": (4, 0.5, 2, 1, 5, 1, 2),
    "stereo_fast_q3_0p5s": (5, 0.5, 2, 0, 3, 0, 0),
    "stereo_q1_b7_0p3s": (6, 0.3, 2, 1, 1, 0, 7),
    "stereo_q4_b8_0p05s": (7, 0.05, 2, 1, 4, 0, 8),
    "mono_q2_one_sample": (8, 1.0 / 44100.0, 1, 1, 2, 0, 0),
    "cfg0_stereo_30s": (0, 30.0, 2, 1, 12, 0, 3),
}
SHORT = [k for k in CASES if k != "cfg0_stereo_30s"]
# Known-token Transformer + range coder cases, the header shapes of the
# reference's Metal known-token test (tests/metal_optimized.cpp:252-270):
# name: (frames, batch, groups, channels, books); tokens (i*73 + 19) % 1024.
KNOWN = {
    "known_17_8_16": (17, 8, 16, 2, 12),
    "known_101_3_1": (101, 3, 1, 2, 12),
    "known_51_3_1": (51, 3, 1, 2, 12),
    "known_35_3_2": (35, 3, 2, 2, 12),
    "known_17_1_1": (17, 1, 1, 2, 12),
    "known_3_8_2": (3, 8, 2, 2, 12),
    "known_1026_1_1": (1026, 1, 1, 2, 1),
    "known_mono_40_2_1": (40, 2, 1, 1, 9),
}


# cfg4 box batch: 30 s joint-stereo clips coded at q=12, batch 3, encode only
# (stream bytes are the contract; decoding a byte-identical stream is checked
# by its token CRC).  Seeds are bench.py's clip seeds rank*100000 + i: clips
# 1..8 of rank 0 and clip 0 of ranks 1..7, so every rank of an 8-GPU bench
# byte-checks at least one clip.
CFG4_SEEDS = list(range(1, 9)) + [r * 100000 for r in range(1, 8)]
CFG4_DIR = HERE / "cfg4"
# cfg3 DAC-only decode: 60 s mono, 9 books, tokens uniform in [0, 1024) from
# seed 3, packed as a fast (method 0) stream and decoded by the reference.
CFG3 = {"seconds": 60.0, "books": 9, "token_seed": 3}


def cfg3_tokens() -> np.ndarray:
    frames = -(-int(round(CFG3["seconds"] * 44100)) // 512)
    rng = np.random.default_rng(CFG3["token_seed"])
    return rng.integers(0, 1024, size=frames * CFG3["books"]).astype(np.uint16)


def run_cfg3(package: pathlib.Path) -> dict:
    lib = ref_library()
    tokens = cfg3_tokens()
    frames = tokens.size // CFG3["books"]
    out = ctypes.POINTER(ctypes.c_uint8)()
    nbytes = ctypes.c_size_t()
    ref_check(lib, lib.ref_pack_fast(1, 1, CFG3["books"], ctypes.c_size_t(frames),
                                     tokens.ctypes.data_as(ctypes.c_void_p), ctypes.byref(out),
                                     ctypes.byref(nbytes)))
    stream = bytes(out[: nbytes.value])
    lib.ref_free(out)
    pcm_out = ctypes.POINTER(ctypes.c_float)()
    ns, nc = ctypes.c_size_t(), ctypes.c_uint()
    t0 = time.time()
    ref_check(lib, lib.ref_decode(str(package).encode(), stream, ctypes.c_size_t(len(stream)),
                                  ctypes.byref(pcm_out), ctypes.byref(ns), ctypes.byref(nc)))
    decode_s = time.time() - t0
    decoded = np.ctypeslib.as_array(pcm_out, shape=(ns.value,)).copy()
    lib.ref_free(pcm_out)
    record = {"case": "cfg3_mono_60s", "frames": frames, "books": CFG3["books"], "channels": 1,
              "method": 0, "tokens": "numpy default_rng(3).integers(0, 1024, frames*books)",
              "weights_seed": 0, "pack_id": tsac_cuda.SEEDED_PACK_ID,
              "stream_bytes": len(stream), "stream_sha256": sha(stream),
              "pcm_samples": int(decoded.size), "pcm_channels": nc.value,
              "pcm_sha256": sha(decoded.astype("<f4").tobytes()),
              "pcm_max_abs": float(np.abs(decoded).max()),
              "pcm_head": decoded[: 4096].astype(float).tolist(),
              "reference_decode_seconds": round(decode_s, 3)}
    (HERE / "cfg3_mono_60s.tsac").write_bytes(stream)
    (HERE / "cfg3_mono_60s.json").write_text(json.dumps(record, indent=1) + "\n")
    return record


def run_cfg4(seed: int) -> dict:
    package = tsac_cuda.seeded_package(0)
    lib = ref_library()
    pcm = synthetic.music_like(seed, 30.0, 2)
    out = ctypes.POINTER(ctypes.c_uint8)()
    nbytes, bits = ctypes.c_size_t(), ctypes.c_size_t()
    t0 = time.time()
    ref_check(lib, lib.ref_encode(str(package).encode(), pcm.ctypes.data_as(ctypes.c_void_p),
                                  ctypes.c_size_t(2), ctypes.c_size_t(pcm.shape[0]), 1, 12, 0, 3,
                                  ctypes.byref(out), ctypes.byref(nbytes), ctypes.byref(bits)))
    encode_s = time.time() - t0
    stream = bytes(out[: nbytes.value])
    lib.ref_free(out)
    record = {"pcm_seed": seed, "seconds": 30.0, "channels": 2, "method": 1, "codebooks": 12,
              "batch": 3, "weights_seed": 0, "pack_id": tsac_cuda.SEEDED_PACK_ID,
              "stream_bytes": len(stream), "stream_sha256": sha(stream),
              "symbol_bits": bits.value, "reference_encode_seconds": round(encode_s, 3)}
    CFG4_DIR.mkdir(exist_ok=True)
    (CFG4_DIR / f"seed_{seed}.json").write_text(json.dumps(record, indent=1) + "\n")
    return record


def known_tokens(frames, groups, books):
    i = np.arange(frames * groups * books, dtype=np.int64)
    return ((i * 73 + 19) % 1024).astype(np.uint16)


def run_known(name: str, package: pathlib.Path) -> dict:
    frames, batch, groups, channels, books = KNOWN[name]
    lib = ref_library()
    tokens = known_tokens(frames, groups, books)
    crc = np.zeros(tokens.size, np.uint32)
    out = ctypes.POINTER(ctypes.c_uint8)()
    nbytes = ctypes.c_size_t()
    t0 = time.time()
    ref_check(lib, lib.ref_pack_normal(str(package).encode(), channels, groups, books,
                                       ctypes.c_size_t(frames), batch,
                                       tokens.ctypes.data_as(ctypes.c_void_p), ctypes.byref(out),
                                       ctypes.byref(nbytes), crc.ctypes.data_as(ctypes.c_void_p)))
    stream = bytes(out[: nbytes.value])
    lib.ref_free(out)
    record = {"case": name, "frames": frames, "batch": batch, "groups": groups,
              "channels": channels, "books": books, "tokens": "(i*73+19)%1024",
              "weights_seed": 0, "stream_bytes": len(stream), "stream_sha256": sha(stream),
              "probability_row_crc32": [int(c) for c in crc],
              "reference_seconds": round(time.time() - t0, 3)}
    (HERE / f"{name}.tsac").write_bytes(stream)
    (HERE / f"{name}.json").write_text(json.dumps(record) + "\n")
    return record


def ref_library() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(REF))
    lib.ref_last_error.restype = ctypes.c_char_p
    return lib


def ref_check(lib, rc):
    if rc != 0:
        raise RuntimeError(lib.ref_last_error().decode())


def sha(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def run_case(name: str, package: pathlib.Path) -> dict:
    seed, seconds, channels, method, codebooks, separate, batch = CASES[name]
    lib = ref_library()
    pcm = synthetic.music_like(seed, seconds, channels)
    samples = pcm.shape[0]
    out = ctypes.POINTER(ctypes.c_uint8)()
    nbytes, bits = ctypes.c_size_t(), ctypes.c_size_t()
    t0 = time.time()
    ref_check(lib, lib.ref_encode(str(package).encode(), pcm.ctypes.data_as(ctypes.c_void_p),
                                  ctypes.c_size_t(channels), ctypes.c_size_t(samples), method,
                                  codebooks, separate, batch, ctypes.byref(out),
                                  ctypes.byref(nbytes), ctypes.byref(bits)))
    encode_s = time.time() - t0
    stream = bytes(out[: nbytes.value])
    lib.ref_free(out)
    tok = ctypes.POINTER(ctypes.c_uint16)()
    count = ctypes.c_size_t()
    ref_check(lib, lib.ref_stream_tokens(str(package).encode(), stream, ctypes.c_size_t(len(stream)),
                                         ctypes.byref(tok), ctypes.byref(count)))
    tokens = np.ctypeslib.as_array(tok, shape=(count.value,)).copy()
    lib.ref_free(tok)
    pcm_out = ctypes.POINTER(ctypes.c_float)()
    ns, nc = ctypes.c_size_t(), ctypes.c_uint()
    t0 = time.time()
    ref_check(lib, lib.ref_decode(str(package).encode(), stream, ctypes.c_size_t(len(stream)),
                                  ctypes.byref(pcm_out), ctypes.byref(ns), ctypes.byref(nc)))
    decode_s = time.time() - t0
    decoded = np.ctypeslib.as_array(pcm_out, shape=(ns.value,)).copy()
    lib.ref_free(pcm_out)
    record = {
        "case": name, "pcm_seed": seed, "seconds": seconds, "channels": channels,
        "method": method, "codebooks": codebooks, "separate": separate, "batch": batch,
        "weights_seed": 0, "pack_id": tsac_cuda.SEEDED_PACK_ID,
        "stream_bytes": len(stream), "stream_sha256": sha(stream),
        "symbol_bits": bits.value if method == 1 else None,
        "tokens": int(tokens.size), "tokens_sha256": sha(tokens.astype("<u2").tobytes()),
        "pcm_samples": int(decoded.size), "pcm_channels": nc.value,
        "pcm_sha256": sha(decoded.astype("<f4").tobytes()),
        "pcm_head": decoded[: 4096].astype(float).tolist(),
        "reference_encode_seconds": round(encode_s, 3),
        "reference_decode_seconds": round(decode_s, 3),
    }
    if len(stream) <= 65536:
        (HERE / f"{name}.tsac").write_bytes(stream)
    (HERE / f"{name}.json").write_text(json.dumps(record, indent=1) + "\n")
    return record


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--cases", default="short",
                        help="'short', 'all', 'known', 'cfg4' or a comma-separated list of case names")
    parser.add_argument("--jobs", type=int, default=1, help="worker processes for 'cfg4'")
    args = parser.parse_args()
    if args.cases == "cfg4":
        tsac_cuda.seeded_package(0)
        todo = [s for s in CFG4_SEEDS if not (CFG4_DIR / f"seed_{s}.json").exists()]
        ctx = multiprocessing.get_context("spawn")
        with concurrent.futures.ProcessPoolExecutor(args.jobs, mp_context=ctx) as pool:
            for r in pool.map(run_cfg4, todo):
                print("cfg4 seed", r["pcm_seed"], r["stream_bytes"], r["stream_sha256"][:16],
                      r["reference_encode_seconds"], flush=True)
        return
    names = SHORT if args.cases == "short" else list(KNOWN) if args.cases == "known" \
        else list(CASES) + list(KNOWN) if args.cases == "all" else args.cases.split(",")
    package = tsac_cuda.seeded_package(0)
    for name in names:
        if name == "cfg3_mono_60s":
            r = run_cfg3(package)
            print(name, r["stream_bytes"], r["pcm_sha256"][:16], r["reference_decode_seconds"],
                  flush=True)
            continue
        if name in KNOWN:
            r = run_known(name, package)
            print(name, r["stream_bytes"], r["stream_sha256"][:16], r["reference_seconds"],
                  flush=True)
            continue
        r = run_case(name, package)
        print(name, r["stream_bytes"], r["stream_sha256"][:16],
              r["reference_encode_seconds"], r["reference_decode_seconds"], flush=True)


if __name__ == "__main__":
    main()
