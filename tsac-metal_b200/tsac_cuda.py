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
import shutil
import threading
import weakref

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
    """Directory of the seeded 20-file package (generated once, then cached).

    Safe under concurrent callers (one process per GPU on a fresh host): an
    exclusive lock on a file beside the cache serialises generation, the
    package is published by renaming a finished directory, and a process that
    waited finds it done."""
    import fcntl

    base = cache_root() / f"seed{seed}"
    package = base / "package"
    marker = package / "weights-manifest.cmake"
    if marker.exists():
        return package
    base.mkdir(parents=True, exist_ok=True)
    with open(base / "generate.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)  # released when the file closes, or the process ends
        if marker.exists():
            return package
        source = base / "source"
        tmp = base / f"package.tmp{os.getpid()}"
        if tmp.exists():
            shutil.rmtree(tmp)
        if package.exists():  # left by an interrupted earlier attempt
            shutil.rmtree(package)
        write_seeded_sources(source, seed)
        pack_models(source, tmp)
        tmp.rename(package)
    return package


# ------------------------------------------------------------ kernel calls --
# Thin wrappers over the per-kernel C-ABI entry points.  Arguments are torch
# CUDA tensors (torch supplies device memory and streams; the arithmetic is
# entirely in this library's kernels).
def _dev(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def qlinear_scratch_bytes(m: int, k: int) -> int:
    lib = library()
    lib.tsac_cuda_qlinear_scratch_bytes.restype = ctypes.c_size_t
    return lib.tsac_cuda_qlinear_scratch_bytes(ctypes.c_size_t(m), ctypes.c_size_t(k))


def qlinear(weights, scales, bias, x, y, scratch, residual=None, error_word=None):
    """y[m][n] = bf16(W x + b) (+residual), all tensors on the device."""
    n, k = weights.shape
    m = x.shape[0]
    check(library().tsac_cuda_qlinear(
        _dev(weights), _dev(scales), _dev(bias), ctypes.c_size_t(k), ctypes.c_size_t(n), _dev(x),
        ctypes.c_size_t(m), _dev(residual), _dev(y), _dev(scratch),
        ctypes.c_size_t(scratch.numel() * scratch.element_size()), _dev(error_word), _stream()))


# --------------------------------------------------------------- analyzer --
@dataclasses.dataclass
class EncodeOptions:
    """tsac::EncodeOptions (include/tsac/audio_analyzer.hpp:16-22)."""
    method: str = "normal"          # "normal" or "fast"
    codebooks: int = 0              # 0: model maximum
    separate_channels: bool = False
    entropy_batch: int | None = None  # None: automatic


class _Options(ctypes.Structure):
    _fields_ = [("method", ctypes.c_int), ("codebooks", ctypes.c_uint),
                ("separate_channels", ctypes.c_int), ("entropy_batch", ctypes.c_int)]


def _options(o: EncodeOptions | None) -> _Options:
    o = o or EncodeOptions()
    if o.method not in ("normal", "fast"):
        raise TsacError("invalid coding method")
    return _Options(1 if o.method == "normal" else 0, o.codebooks,
                    1 if o.separate_channels else 0, o.entropy_batch or 0)


@dataclasses.dataclass
class PcmAudio:
    """tsac::PcmAudio: interleaved float32 samples [frames][channels]."""
    samples: np.ndarray
    channels: int


def _adopt(ptr, count, dtype):
    """A numpy view of a library-allocated buffer that frees it (tsac_cuda_free)
    when the last array using it is collected: large results (decoded PCM) are
    not copied a second time."""
    lib = library()
    if not count:
        lib.tsac_cuda_free(ptr)
        return np.zeros(0, dtype)
    address = ptr.value if isinstance(ptr, ctypes.c_void_p) else int(ptr)
    storage = (np.ctypeslib.as_ctypes_type(dtype) * count).from_address(address)
    weakref.finalize(storage, lib.tsac_cuda_free, ctypes.c_void_p(address))
    return np.frombuffer(storage, dtype)


def _take(ptr, count, dtype):
    """Copy a library-allocated buffer into numpy and free it."""
    lib = library()
    if count:
        arr = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(np.ctypeslib.as_ctypes_type(dtype))),
                                    shape=(count,)).copy()
    else:
        arr = np.zeros(0, dtype)
    lib.tsac_cuda_free(ptr)
    return arr


class CudaAnalyzer:
    """B200 implementation of tsac::AudioAnalyzer (include/tsac/audio_analyzer.hpp:30-37).

    Calls are synchronous; one instance is used by one thread at a time.
    """

    def __init__(self, package: os.PathLike, device: int = 0):
        lib = library()
        self._ctx = ctypes.c_void_p()
        check(lib.tsac_cuda_context_create(str(package).encode(), device, ctypes.byref(self._ctx)))

    def set_exact_synthesis(self, exact: bool) -> None:
        """Exact (bit-identical PCM) or tensor-core (within tolerance) synthesis."""
        check(library().tsac_cuda_set_exact_synthesis(self._ctx, 1 if exact else 0))

    def set_host_threads(self, threads: int) -> None:
        """Host range-coding worker budget (0: automatic, at most 256), the
        thread count AppleArmAnalyzer takes (src/apple-arm/audio_analyzer.cpp:93)."""
        if threads < 0:
            raise TsacError("invalid thread count")
        check(library().tsac_cuda_set_host_threads(self._ctx, ctypes.c_uint(threads)))

    def set_fast_analysis(self, margin: float) -> None:
        """Certified fast analysis: 0 = exact analysis; margin > 0 = fused
        multiply-add analysis with every frame whose RVQ decision lead is below
        `margin` recomputed exactly (streams stay the reference's)."""
        check(library().tsac_cuda_set_fast_analysis(self._ctx, ctypes.c_float(margin)))

    def fast_analysis_stats(self):
        """(central frames coded, frames flagged uncertain, frames recomputed exactly)."""
        f, u, r = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        check(library().tsac_cuda_fast_analysis_stats(self._ctx, ctypes.byref(f), ctypes.byref(u),
                                                      ctypes.byref(r)))
        return f.value, u.value, r.value

    def close(self):
        if self._ctx:
            library().tsac_cuda_context_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, pcm: np.ndarray, options: EncodeOptions | None = None,
               with_bits: bool = False):
        """pcm: float32 [samples][channels] (interleaved) or any 2-D strided view."""
        pcm = np.asarray(pcm, dtype=np.float32)
        if pcm.ndim == 1:
            pcm = pcm[:, None]
        samples, channels = pcm.shape
        out = ctypes.c_void_p()
        nbytes, bits = ctypes.c_size_t(), ctypes.c_size_t()
        opts = _options(options)
        check(library().tsac_cuda_encode(
            self._ctx, pcm.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(channels),
            ctypes.c_size_t(samples), ctypes.c_ssize_t(pcm.strides[1] // 4),
            ctypes.c_ssize_t(pcm.strides[0] // 4), ctypes.byref(opts), ctypes.byref(out),
            ctypes.byref(nbytes), ctypes.byref(bits)))
        data = _take(out, nbytes.value, np.uint8).tobytes()
        return (data, bits.value) if with_bits else data

    def encode_symbol_bits(self, pcm: np.ndarray, options: EncodeOptions | None = None):
        """encode() plus each symbol's bits in entropy order (what an
        EntropyObserver's after_symbol receives); an empty array for fast streams."""
        pcm = np.asarray(pcm, dtype=np.float32)
        if pcm.ndim == 1:
            pcm = pcm[:, None]
        samples, channels = pcm.shape
        out, per_symbol = ctypes.c_void_p(), ctypes.c_void_p()
        nbytes, count = ctypes.c_size_t(), ctypes.c_size_t()
        opts = _options(options)
        check(library().tsac_cuda_encode_symbol_bits(
            self._ctx, pcm.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(channels),
            ctypes.c_size_t(samples), ctypes.c_ssize_t(pcm.strides[1] // 4),
            ctypes.c_ssize_t(pcm.strides[0] // 4), ctypes.byref(opts), ctypes.byref(out),
            ctypes.byref(nbytes), ctypes.byref(per_symbol), ctypes.byref(count)))
        data = _take(out, nbytes.value, np.uint8).tobytes()
        return data, _take(per_symbol, count.value, np.uint32)

    def decode(self, stream: bytes) -> PcmAudio:
        out = ctypes.c_void_p()
        samples, channels = ctypes.c_size_t(), ctypes.c_uint()
        check(library().tsac_cuda_decode(self._ctx, stream, ctypes.c_size_t(len(stream)),
                                         ctypes.byref(out), ctypes.byref(samples),
                                         ctypes.byref(channels)))
        data = _adopt(out, samples.value, np.float32)
        return PcmAudio(data.reshape(-1, channels.value), channels.value)

    def encode_batch(self, pcms, options: EncodeOptions | None = None):
        pcms = [np.ascontiguousarray(p, dtype=np.float32).reshape(p.shape[0], -1) for p in pcms]
        n = len(pcms)
        ptrs = (ctypes.c_void_p * n)(*[p.ctypes.data for p in pcms])
        chans = (ctypes.c_size_t * n)(*[p.shape[1] for p in pcms])
        sams = (ctypes.c_size_t * n)(*[p.shape[0] for p in pcms])
        outs = (ctypes.c_void_p * n)()
        sizes = (ctypes.c_size_t * n)()
        opts = _options(options)
        check(library().tsac_cuda_encode_batch(self._ctx, ctypes.c_size_t(n), ptrs, chans, sams,
                                               ctypes.byref(opts), outs, sizes))
        return [_take(ctypes.c_void_p(outs[i]), sizes[i], np.uint8).tobytes() for i in range(n)]

    def decode_batch(self, streams):
        n = len(streams)
        bufs = [ctypes.create_string_buffer(s, len(s)) for s in streams]
        ptrs = (ctypes.c_void_p * n)(*[ctypes.addressof(b) for b in bufs])
        sizes = (ctypes.c_size_t * n)(*[len(s) for s in streams])
        outs = (ctypes.c_void_p * n)()
        samples = (ctypes.c_size_t * n)()
        chans = (ctypes.c_uint * n)()
        check(library().tsac_cuda_decode_batch(self._ctx, ctypes.c_size_t(n), ptrs, sizes, outs,
                                               samples, chans))
        return [PcmAudio(_adopt(ctypes.c_void_p(outs[i]), samples[i], np.float32)
                         .reshape(-1, chans[i]), chans[i]) for i in range(n)]

    # ---- pipeline stages (parity tests) ---------------------------------
    def analyze_tokens(self, pcm: np.ndarray, options: EncodeOptions | None = None):
        pcm = np.ascontiguousarray(pcm, dtype=np.float32).reshape(pcm.shape[0], -1)
        out = ctypes.c_void_p()
        count = ctypes.c_size_t()
        opts = _options(options)
        check(library().tsac_cuda_analyze_tokens(
            self._ctx, pcm.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(pcm.shape[1]),
            ctypes.c_size_t(pcm.shape[0]), ctypes.byref(opts), ctypes.byref(out),
            ctypes.byref(count)))
        return _take(out, count.value, np.uint16)

    def dac_analysis(self, channels: int, pcm: np.ndarray) -> np.ndarray:
        pcm = np.ascontiguousarray(pcm, dtype=np.float32)
        frames = pcm.size // channels
        latent = np.zeros((frames // 512, 1024), np.float32)
        check(library().tsac_cuda_dac_analysis(self._ctx, channels, pcm.ctypes.data_as(ctypes.c_void_p),
                                                ctypes.c_size_t(frames),
                                                latent.ctypes.data_as(ctypes.c_void_p)))
        return latent

    def dac_synthesis(self, channels: int, latent: np.ndarray) -> np.ndarray:
        latent = np.ascontiguousarray(latent, dtype=np.float32)
        frames = latent.size // 1024
        pcm = np.zeros((frames * 512, channels), np.float32)
        check(library().tsac_cuda_dac_synthesis(self._ctx, channels,
                                                 latent.ctypes.data_as(ctypes.c_void_p),
                                                 ctypes.c_size_t(frames),
                                                 pcm.ctypes.data_as(ctypes.c_void_p)))
        return pcm

    def rvq_encode(self, channels: int, books: int, latent: np.ndarray) -> np.ndarray:
        latent = np.ascontiguousarray(latent, dtype=np.float32)
        frames = latent.size // 1024
        tokens = np.zeros((frames, books), np.uint16)
        check(library().tsac_cuda_rvq_encode(self._ctx, channels, books,
                                             latent.ctypes.data_as(ctypes.c_void_p),
                                             ctypes.c_size_t(frames),
                                             tokens.ctypes.data_as(ctypes.c_void_p)))
        return tokens

    def rvq_decode(self, channels: int, books: int, tokens: np.ndarray) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint16)
        frames = tokens.size // books
        latent = np.zeros((frames, 1024), np.float32)
        check(library().tsac_cuda_rvq_decode(self._ctx, channels, books,
                                             tokens.ctypes.data_as(ctypes.c_void_p),
                                             ctypes.c_size_t(frames),
                                             latent.ctypes.data_as(ctypes.c_void_p)))
        return latent

    def transformer_probabilities(self, channels, groups, books, frames, batch, tokens,
                                  probabilities=True):
        tokens = np.ascontiguousarray(tokens, dtype=np.uint16)
        symbols = frames * groups * books
        probs = np.zeros((symbols, 1024), np.float32) if probabilities else None
        q15 = np.zeros((symbols, 10), np.uint16)
        check(library().tsac_cuda_transformer_probabilities(
            self._ctx, channels, groups, books, ctypes.c_size_t(frames), batch,
            tokens.ctypes.data_as(ctypes.c_void_p),
            probs.ctypes.data_as(ctypes.c_void_p) if probs is not None else None,
            q15.ctypes.data_as(ctypes.c_void_p)))
        return probs, q15

    def pack_normal(self, channels, groups, books, frames, batch, tokens) -> bytes:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint16)
        out = ctypes.c_void_p()
        nbytes = ctypes.c_size_t()
        check(library().tsac_cuda_pack_normal(self._ctx, channels, groups, books,
                                              ctypes.c_size_t(frames), batch,
                                              tokens.ctypes.data_as(ctypes.c_void_p),
                                              ctypes.byref(out), ctypes.byref(nbytes)))
        return _take(out, nbytes.value, np.uint8).tobytes()


def stream_info(stream: bytes):
    """(channels, samples_per_channel, symbols) of a .tsac stream."""
    ch, spc, sym = ctypes.c_uint(), ctypes.c_size_t(), ctypes.c_size_t()
    check(library().tsac_cuda_stream_info(stream, ctypes.c_size_t(len(stream)), ctypes.byref(ch),
                                          ctypes.byref(spc), ctypes.byref(sym)))
    return ch.value, spc.value, sym.value


def unpack_fast(stream: bytes) -> np.ndarray:
    """Token indices of a fast-method stream (header and CRC checked)."""
    ptr, n = ctypes.POINTER(ctypes.c_uint16)(), ctypes.c_size_t()
    check(library().tsac_cuda_unpack_fast(stream, ctypes.c_size_t(len(stream)), ctypes.byref(ptr),
                                          ctypes.byref(n)))
    return _take(ptr, n.value, np.uint16)


def token_crc32(tokens) -> int:
    """CRC-32 (polynomial 0x04c11db7) of token indices, as a normal header stores it."""
    t = np.ascontiguousarray(tokens, dtype=np.uint16)
    fn = library().tsac_cuda_token_crc32
    fn.restype = ctypes.c_uint32
    return fn(t.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(t.size))


def encode_batch_device(analyzer: "CudaAnalyzer", pcm_tensors, options: EncodeOptions | None = None):
    """Encode HBM-resident interleaved PCM (torch CUDA float32 [samples][channels])."""
    n = len(pcm_tensors)
    ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in pcm_tensors])
    chans = (ctypes.c_size_t * n)(*[t.shape[1] for t in pcm_tensors])
    sams = (ctypes.c_size_t * n)(*[t.shape[0] for t in pcm_tensors])
    outs = (ctypes.c_void_p * n)()
    sizes = (ctypes.c_size_t * n)()
    opts = _options(options)
    check(library().tsac_cuda_encode_batch_device(analyzer._ctx, ctypes.c_size_t(n), ptrs, chans,
                                                  sams, ctypes.byref(opts), outs, sizes))
    return [_take(ctypes.c_void_p(outs[i]), sizes[i], np.uint8).tobytes() for i in range(n)]


def decode_batch_device(analyzer: "CudaAnalyzer", streams, out_tensors):
    """Decode into HBM-resident PCM tensors (torch CUDA float32, channels x samples each)."""
    n = len(streams)
    bufs = [ctypes.create_string_buffer(s, len(s)) for s in streams]
    ptrs = (ctypes.c_void_p * n)(*[ctypes.addressof(b) for b in bufs])
    sizes = (ctypes.c_size_t * n)(*[len(s) for s in streams])
    outs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in out_tensors])
    check(library().tsac_cuda_decode_batch_device(analyzer._ctx, ctypes.c_size_t(n), ptrs, sizes,
                                                  outs))
