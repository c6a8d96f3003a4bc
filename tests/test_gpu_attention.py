"""cfg2: the causal attention kernel alone on the GPU vs the oracle, bit for bit.

The oracle is oracle_attention (oracle/oracle.c), a restatement of
scalar::Attention (src/scalar/attention.cpp:12-131) pinned to the reference's
attention checksum and to the reference itself (tests/test_oracle.py).
Shapes follow the cfg2 microbenchmark: 4 heads x 128, batch 3 (three
independent key sequences), Q/K/V ~ N(0, 1) rounded to bf16, seed 2, and
  - decode: one query per lane over T keys, value sums rounded when T > 64;
  - replay decode: the same with rounding forced (the reference rounds a
    replayed context, `time > 64 || prefill`, :128);
  - causal prefill: T queries per lane, query t over keys [0, t], rounded;
for T in {1, 2, 63, 64, 65, 862, 1023, 1024} (the model's temporal range,
capped at 1024 by src/common/cpu_transformer.tpp:321), the codebook range
1..12, and the 62,016-key stress length (12 books x 2 channels x 2584 frames)
that the scalar kernel accepts although the model never produces it.
"""
import ctypes

import numpy as np
import pytest

from support import bf16, oracle, ptr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import tsac_cuda  # noqa: E402

WIDTH = 512
LANES = 3


def _sequences(T, seed=2):
    rng = np.random.default_rng(seed * 100003 + T)
    q = bf16(rng.standard_normal((LANES, T, WIDTH)).astype(np.float32))
    k = bf16(rng.standard_normal((LANES, T, WIDTH)).astype(np.float32))
    v = bf16(rng.standard_normal((LANES, T, WIDTH)).astype(np.float32))
    return q, k, v


def _gpu(queries, meta, keys, values, max_time):
    dev = torch.device("cuda")
    lib = tsac_cuda.library()
    lib.tsac_cuda_attention_scratch_bytes.restype = ctypes.c_size_t
    rows = queries.shape[0]
    tq = torch.from_numpy(queries.view(np.int16)).to(dev)
    tk = torch.from_numpy(keys.reshape(-1, WIDTH).view(np.int16)).to(dev)
    tv = torch.from_numpy(values.reshape(-1, WIDTH).view(np.int16)).to(dev)
    tm = torch.from_numpy(np.ascontiguousarray(meta, dtype=np.int32)).to(dev)
    out = torch.full((rows, WIDTH), -1, dtype=torch.int16, device=dev)
    nbytes = lib.tsac_cuda_attention_scratch_bytes(ctypes.c_size_t(rows), ctypes.c_size_t(max_time))
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    d = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    tsac_cuda.check(lib.tsac_cuda_attention(d(tq), d(tm), d(tk), d(tv), ctypes.c_size_t(rows),
                                            ctypes.c_size_t(max_time), d(out), d(scratch),
                                            ctypes.c_size_t(nbytes),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


def _oracle(query, keys, values, time, prefill):
    y = np.zeros(WIDTH, np.uint16)
    oracle().oracle_attention(ptr(np.ascontiguousarray(query)), ptr(np.ascontiguousarray(keys[:time])),
                              ptr(np.ascontiguousarray(values[:time])), 4, 128, time, int(prefill), ptr(y))
    return y


def _decode(T, force_round):
    q, k, v = _sequences(T)
    queries = np.ascontiguousarray(q[:, -1])
    meta = [(0, lane * T, T, -1, int(force_round or T > 64)) for lane in range(LANES)]
    got = _gpu(queries, meta, k, v, T)
    for lane in range(LANES):
        want = _oracle(queries[lane], k[lane], v[lane], T, force_round)
        assert np.array_equal(got[lane], want), f"lane {lane} T={T}"


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 862, 1023, 1024])
def test_decode_matches_oracle(T):
    _decode(T, force_round=False)


@pytest.mark.parametrize("T", [1, 40, 64, 65, 256, 1024])
def test_replay_rounded_decode_matches_oracle(T):
    _decode(T, force_round=True)


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 862, 1023, 1024])
def test_causal_prefill_matches_oracle(T):
    q, k, v = _sequences(T)
    queries = q.reshape(LANES * T, WIDTH)
    meta = [(0, lane * T, t + 1, -1, 1) for lane in range(LANES) for t in range(T)]
    got = _gpu(queries, meta, k, v, T)
    rng = np.random.default_rng(T)
    # Every row for short sequences; a seeded sample of rows (always the block
    # edges) for long ones, to keep the C oracle to a few seconds.
    picks = range(T) if T <= 128 else sorted(set(rng.choice(T, 48, replace=False).tolist())
                                             | {0, 63, 64, 65, T - 1})
    for lane in range(LANES):
        for t in picks:
            want = _oracle(q[lane, t], k[lane], v[lane], t + 1, True)
            assert np.array_equal(got[lane * T + t], want), f"lane {lane} t={t} T={T}"


def test_codebook_lengths_match_oracle():
    """The codebook stack's histories: 1..12 keys, never rounded."""
    for T in range(1, 13):
        _decode(T, force_round=False)


def test_stress_length_62016_keys():
    _decode(12 * 2 * 2584, force_round=False)


def test_rows_share_one_launch_with_mixed_lengths():
    """Rows of different history lengths (1 block, several blocks, partial last
    block) in one call, as a decode step batches lanes of different ages."""
    T = 300
    q, k, v = _sequences(T, seed=5)
    times = [1, 64, 65, 130, 299, 300]
    meta = [(0, (i % LANES) * T, t, -1, int(t > 64)) for i, t in enumerate(times)]
    queries = np.stack([q[i % LANES, t - 1] for i, t in enumerate(times)])
    got = _gpu(queries, meta, k, v, T)
    for i, t in enumerate(times):
        lane = i % LANES
        assert np.array_equal(got[i], _oracle(queries[i], k[lane], v[lane], t, False)), f"time {t}"
