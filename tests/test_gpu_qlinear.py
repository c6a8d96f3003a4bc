"""Quantized linear (BF8L) on the GPU vs the oracle: bit-exact bf16 outputs.

Shapes: every projection shape of the model contract (src/models/contract.cpp:88-110)
and the cfg1 microbench shapes with M in {1, 3, 16, 64, 256}; plus edge rows
(all-zero columns, huge/small magnitudes, subnormal inputs) and the fused
residual epilogue.
"""
import numpy as np
import pytest

from support import bf16, f32, oracle, ptr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402


def _case(k, n, m, seed, special=False):
    rng = np.random.default_rng(seed)
    w = rng.integers(-128, 128, size=(n, k), dtype=np.int8)
    ws = (rng.uniform(0.5, 2.0, size=(k // 256, n)) / 127).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32)
    x = bf16(rng.standard_normal((m, k)).astype(np.float32))
    if special and m >= 4:
        x[0] = 0
        x[1] = bf16(rng.standard_normal(k).astype(np.float32) * np.float32(1e30))
        x[2] = bf16(rng.standard_normal(k).astype(np.float32) * np.float32(1e-39))
        x[3, :128] = bf16(np.float32(1e-40))
    return w, ws, b, x


def _run_gpu(w, ws, b, x, residual=None):
    dev = torch.device("cuda")
    n, k = w.shape
    m = x.shape[0]
    tw = torch.from_numpy(w).to(dev)
    ts = torch.from_numpy(ws).to(dev)
    tb = torch.from_numpy(b).to(dev)
    tx = torch.from_numpy(x.view(np.int16)).to(dev)
    ty = torch.empty((m, n), dtype=torch.int16, device=dev)
    tr = torch.from_numpy(residual.view(np.int16)).to(dev) if residual is not None else None
    scratch = torch.empty(tsac_cuda.qlinear_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    tsac_cuda.qlinear(tw, ts, tb, tx, ty, scratch, residual=tr, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return ty.cpu().numpy().view(np.uint16)


def _run_oracle(w, ws, b, x):
    n, k = w.shape
    m = x.shape[0]
    y = np.zeros((m, n), np.uint16)
    oracle().oracle_linear(ptr(np.ascontiguousarray(w)), ptr(ws), ptr(b), k, n, ptr(x), m, ptr(y))
    return y


MODEL_SHAPES = [(512, 1536), (512, 512), (512, 2048), (2048, 512), (1024, 512), (512, 1024)]


@pytest.mark.parametrize("k,n", MODEL_SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 6, 8, 14, 16, 24, 96, 130])
def test_model_shapes_bit_exact(k, n, m):
    w, ws, b, x = _case(k, n, m, seed=k * 7 + n + m, special=True)
    assert np.array_equal(_run_gpu(w, ws, b, x), _run_oracle(w, ws, b, x))


@pytest.mark.parametrize("k,n", [(1024, 1024), (1024, 4096), (4096, 1024)])
@pytest.mark.parametrize("m", [1, 3, 16, 64, 256])
def test_cfg1_shapes_bit_exact(k, n, m):
    w, ws, b, x = _case(k, n, m, seed=m + n)
    assert np.array_equal(_run_gpu(w, ws, b, x), _run_oracle(w, ws, b, x))


@pytest.mark.parametrize("k,n", MODEL_SHAPES)
@pytest.mark.parametrize("m", [256, 257, 383, 1000])
def test_gemm_model_shapes_bit_exact(k, n, m):
    """From 256 rows the tcgen05 int8 GEMM runs (qlinear_tc.cu): full and
    partial 128-row tiles, every model projection shape, edge-value rows."""
    w, ws, b, x = _case(k, n, m, seed=k * 3 + n + m, special=True)
    assert np.array_equal(_run_gpu(w, ws, b, x), _run_oracle(w, ws, b, x))


@pytest.mark.parametrize("k,n", [(1024, 1024), (1024, 4096), (4096, 1024)])
def test_gemm_cfg1_shapes_bit_exact(k, n):
    w, ws, b, x = _case(k, n, 512, seed=k + n)
    assert np.array_equal(_run_gpu(w, ws, b, x), _run_oracle(w, ws, b, x))


@pytest.mark.parametrize("m", [3, 40, 300])
def test_residual_epilogue(m):
    w, ws, b, x = _case(512, 512, m, seed=99)
    rng = np.random.default_rng(5)
    res = bf16(rng.standard_normal((m, 512)).astype(np.float32))
    base = _run_oracle(w, ws, b, x)
    expected = bf16(f32(res) + f32(base))
    assert np.array_equal(_run_gpu(w, ws, b, x, residual=res), expected)


def test_nonfinite_input_sets_error_word():
    w, ws, b, x = _case(512, 64, 2, seed=3)
    x[1, 7] = 0x7F80  # +inf
    dev = torch.device("cuda")
    scratch = torch.empty(tsac_cuda.qlinear_scratch_bytes(2, 512), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    y = torch.empty((2, 64), dtype=torch.int16, device=dev)
    tsac_cuda.qlinear(torch.from_numpy(w).to(dev), torch.from_numpy(ws).to(dev),
                      torch.from_numpy(b).to(dev), torch.from_numpy(x.view(np.int16)).to(dev), y,
                      scratch, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1


def test_rejects_bad_shapes():
    dev = torch.device("cuda")
    w = torch.zeros((64, 300), dtype=torch.int8, device=dev)
    s = torch.zeros((1, 64), dtype=torch.float32, device=dev)
    b = torch.zeros(64, dtype=torch.float32, device=dev)
    x = torch.zeros((1, 300), dtype=torch.int16, device=dev)
    y = torch.zeros((1, 64), dtype=torch.int16, device=dev)
    scratch = torch.zeros(4096, dtype=torch.uint8, device=dev)
    with pytest.raises(tsac_cuda.TsacError):
        tsac_cuda.qlinear(w, s, b, x, y, scratch)
