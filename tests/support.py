"""Shared test plumbing: ctypes handles on the oracle libraries.

oracle/liboracle.so  — this repository's C restatement (always buildable).
oracle/_ref/libtsac_ref.so — the reference scalar path compiled from its own
sources (built here by oracle/Makefile; it travels with the tree to the GPU
box).  Tests that need it skip when it is absent.
"""
from __future__ import annotations

import ctypes
import functools
import pathlib
import subprocess

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
ORACLE = ROOT / "oracle" / "liboracle.so"
REF = ROOT / "oracle" / "_ref" / "libtsac_ref.so"
GOLDEN = ROOT / "tests" / "golden"

c_void_p, c_size_t = ctypes.c_void_p, ctypes.c_size_t


def ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


@functools.lru_cache(None)
def oracle() -> ctypes.CDLL:
    if not ORACLE.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "oracle"], check=True,
                       stdout=subprocess.DEVNULL)
    lib = ctypes.CDLL(str(ORACLE))
    lib.oracle_bf16.restype = ctypes.c_uint16
    lib.oracle_bf16.argtypes = [ctypes.c_float]
    lib.oracle_float.restype = ctypes.c_float
    lib.oracle_float.argtypes = [ctypes.c_uint16]
    lib.oracle_exp.restype = ctypes.c_float
    lib.oracle_exp.argtypes = [ctypes.c_float]
    lib.oracle_probability_sum.restype = ctypes.c_float
    lib.oracle_probability_sum.argtypes = [c_void_p, c_size_t]
    lib.oracle_bisection_masses.argtypes = [c_void_p, c_size_t, c_void_p]
    lib.oracle_conditional_q15.restype = ctypes.c_uint16
    lib.oracle_conditional_q15.argtypes = [ctypes.c_float, ctypes.c_float]
    lib.oracle_gelu.restype = ctypes.c_uint16
    lib.oracle_gelu.argtypes = [ctypes.c_uint16]
    lib.oracle_rvq_nearest.restype = ctypes.c_uint16
    lib.oracle_conv1d.restype = c_size_t
    lib.oracle_conv1d.argtypes = [c_size_t] * 6 + [ctypes.c_int] + [c_void_p] * 3 + [c_size_t, c_void_p]
    lib.oracle_categorical_path.restype = c_size_t
    lib.oracle_categorical_path.argtypes = [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]
    lib.oracle_linear.argtypes = [c_void_p] * 3 + [c_size_t] * 2 + [c_void_p, c_size_t, c_void_p]
    lib.oracle_attention.argtypes = [c_void_p] * 3 + [c_size_t] * 3 + [ctypes.c_int, c_void_p]
    lib.oracle_layer_norm.argtypes = [c_void_p] * 3 + [c_size_t, c_void_p]
    lib.oracle_rotary.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.oracle_softmax.argtypes = [c_void_p, c_size_t, c_void_p]
    lib.oracle_snake.argtypes = [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]
    lib.oracle_bf8l.argtypes = [c_void_p, c_size_t, c_void_p, c_void_p]
    lib.oracle_rvq_project.argtypes = [ctypes.c_uint16, c_void_p, c_void_p, c_void_p, c_void_p]
    return lib


def ref_available() -> bool:
    return REF.exists()


@functools.lru_cache(None)
def ref() -> ctypes.CDLL:
    if not REF.exists():
        pytest.skip("reference oracle oracle/_ref/libtsac_ref.so not built")
    lib = ctypes.CDLL(str(REF))
    lib.ref_last_error.restype = ctypes.c_char_p
    lib.ref_gelu.restype = ctypes.c_uint16
    lib.ref_gelu.argtypes = [ctypes.c_uint16]
    lib.ref_probability_sum.restype = ctypes.c_float
    lib.ref_probability_sum.argtypes = [c_void_p, c_size_t]
    lib.ref_original_exp.restype = ctypes.c_float
    lib.ref_original_exp.argtypes = [ctypes.c_float]
    lib.ref_conditional_q15.restype = ctypes.c_uint16
    lib.ref_conditional_q15.argtypes = [ctypes.c_float, ctypes.c_float]
    return lib


def ref_check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(ref().ref_last_error().decode())


def bf16(x: np.ndarray) -> np.ndarray:
    """Integer round-to-nearest-even float32 -> bf16 bits (the codec's rule)."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
