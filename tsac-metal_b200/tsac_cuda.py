"""Python binding of libtsac_cuda.so (the C ABI declared in include/tsac_cuda.h).

Mirrors the reference's public analyzer API (include/tsac/audio_analyzer.hpp):
`CudaAnalyzer(package).encode(pcm, EncodeOptions) -> bytes` and
`.decode(stream) -> PcmAudio`, with tsac::Error surfacing as `TsacError`.
There is no CPU fallback: loading fails loudly if the library is missing, and
every GPU entry point fails with TSAC_CUDA_ERROR_DEVICE without a device.
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
import pathlib
import threading

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIBRARY = HERE / "libtsac_cuda.so"
# Pack ID of every seeded package this library writes (16 lowercase hex digits,
# as the reference packer requires, src/weights/pack_main.cpp:748-751).
SEEDED_PACK_ID = "b200b200b200b200"

OK, ERROR, ERROR_DEVICE, ERROR_NUMERIC = 0, 1, 2, 3


class TsacError(RuntimeError):
    """tsac::Error equivalent; `.status` holds the C-ABI status code."""

    def __init__(self, message: str, status: int = ERROR):
        super().__init__(message)
        self.status = status


_lib = None
_lock = threading.Lock()


def library() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise TsacError(
                    f"{LIBRARY} is missing; build it with `make -C {HERE}` "
                    "(there is no CPU fallback)", ERROR_DEVICE)
            lib = ctypes.CDLL(str(LIBRARY))
            lib.tsac_cuda_last_error.restype = ctypes.c_char_p
            _lib = lib
        return _lib


def check(status: int) -> None:
    if status != OK:
        message = library().tsac_cuda_last_error().decode("utf-8", "replace")
        raise TsacError(message, status)


# ---------------------------------------------------------------- packages --
def write_seeded_sources(directory: os.PathLike, seed: int) -> None:
    check(library().tsac_cuda_write_seeded_sources(
        str(directory).encode(), ctypes.c_uint64(seed)))


def pack_models(source: os.PathLike, output: os.PathLike, pack_id: str = SEEDED_PACK_ID,
                include_transformer: bool = True) -> None:
    check(library().tsac_cuda_pack_models(
        str(source).encode(), str(output).encode(), pack_id.encode(),
        1 if include_transformer else 0))


def cache_root() -> pathlib.Path:
    root = os.environ.get("TSAC_B200_CACHE")
    return pathlib.Path(root) if root else pathlib.Path("/tmp/tsac_b200_models")


def seeded_package(seed: int = 0) -> pathlib.Path:
    """Directory of the seeded 20-file package (generated once, then cached)."""
    package = cache_root() / f"seed{seed}" / "package"
    marker = package / "weights-manifest.cmake"
    if marker.exists():
        return package
    source = cache_root() / f"seed{seed}" / "source"
    tmp = package.with_name(f"package.tmp{os.getpid()}")
    write_seeded_sources(source, seed)
    pack_models(source, tmp)
    if not marker.exists():
        tmp.rename(package)
    return package
