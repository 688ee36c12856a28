"""GPU parity of the grouped-query attention kernels and the KV-cache append.

The reference has no attention operator (it is a planned primitive,
docs/roadmap.md:58-60), so the oracle is the standard definition in float64
(``checker.gqa_attention_f64``) on the same seeded inputs.  Bounds:
* KV-cache append: bit-exact (a copy); out-of-range slots are skipped and
  flagged;
* attention outputs (f16): normwise max error <= 1e-3 and element-wise
  error with an rms floor <= 2e-3 against float64 -- the f16 output rounding
  is up to 4.9e-4, the softmax uses the hardware exp2 approximation
  (relative error ~2^-22) and f32 accumulation;
* prefill (tensor cores): the probabilities P are rounded to f16 before the
  P.V contraction (as in FlashAttention; the same class of error as the
  Q4_0 prefill GEMM's f16 weights), so over long rows the rms-floored
  element-wise error reaches ~3e-3 (2048 positions); its bound is 4e-3,
  the normwise bound stays 1e-3.

Shapes: Llama-3.2-1B's attention (32 query heads, 8 KV heads, head_dim 64)
and Llama-3-8B's (32 / 8, head_dim 128) at decode with context lengths from
1 to 8192 (one and many position chunks per sequence, ragged final tiles),
batches of sequences with different lengths (including 0), and the
multi-head-attention (group 1) and 8-query-heads-per-KV-head extremes.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import errors, ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain  # noqa: E402

NORMWISE = 1e-3
ELEMENTWISE = 2e-3
PREFILL_ELEMENTWISE = 4e-3


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def test_kv_cache_append_is_a_copy_and_flags_bad_slots(ctx):
    rng = np.random.default_rng(3)
    rows, kvh, hd, tokens = 64, 8, 64, 5
    kc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    vc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    kn = f16(rng.normal(0, 1, (tokens, kvh, hd)))
    vn = f16(rng.normal(0, 1, (tokens, kvh, hd)))
    slots = np.array([3, 63, 0, 17, 40], np.int32)
    t = {n: ctx.from_bytes(plain(a.shape, DType.F16), a) for n, a in
         (("kc", kc), ("vc", vc), ("kn", kn), ("vn", vn))}
    st = ctx.from_bytes(plain((tokens,), DType.I32), slots)
    ops.kv_cache_append_f16(ctx, t["kn"], t["vn"], t["kc"], t["vc"], st)
    want_k, want_v = kc.copy(), vc.copy()
    want_k[slots], want_v[slots] = kn, vn
    got_k = np.frombuffer(ctx.read_bytes(t["kc"]), np.float16).reshape(rows, kvh, hd)
    got_v = np.frombuffer(ctx.read_bytes(t["vc"]), np.float16).reshape(rows, kvh, hd)
    assert np.array_equal(got_k.view(np.uint16), want_k.view(np.uint16))
    assert np.array_equal(got_v.view(np.uint16), want_v.view(np.uint16))
    # slots outside the cache: skipped, flagged
    bad = ctx.from_bytes(plain((tokens,), DType.I32), np.array([1, -1, 64, 2, 9], np.int32))
    with pytest.raises(errors.IndexOutOfRange):
        ops.kv_cache_append_f16(ctx, t["kn"], t["vn"], t["kc"], t["vc"], bad)
    got_k = np.frombuffer(ctx.read_bytes(t["kc"]), np.float16).reshape(rows, kvh, hd)
    want_k[[1, 2, 9]] = kn[[0, 3, 4]]
    assert np.array_equal(got_k.view(np.uint16), want_k.view(np.uint16))
    assert ctx.device_status() == 0


def _decode_case(ctx, batch, qh, kvh, hd, lens, capacity, seed, max_len=None):
    rng = np.random.default_rng(seed)
    rows = batch * capacity
    kc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    vc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    q = f16(rng.normal(0, 1, (batch, qh, hd)))
    lens = np.asarray(lens, np.int32)
    max_len = int(max(lens.max(), 1)) if max_len is None else max_len
    tq = ctx.from_bytes(plain(q.shape, DType.F16), q)
    tk = ctx.from_bytes(plain(kc.shape, DType.F16), kc)
    tv = ctx.from_bytes(plain(vc.shape, DType.F16), vc)
    tl = ctx.from_bytes(plain((batch,), DType.I32), lens)
    to = ctx.from_bytes(plain(q.shape, DType.F16), np.full(q.shape, np.nan, np.float16))
    ops.gqa_attention_decode_f16(ctx, tq, tk, tv, tl, to, capacity, max_len)
    got = np.frombuffer(ctx.read_bytes(to), np.float16).astype(np.float32).reshape(q.shape)
    assert ctx.device_status() == 0
    scale = 1.0 / math.sqrt(hd)
    for b in range(batch):
        n = min(int(lens[b]), max_len)
        if n == 0:
            assert np.all(got[b] == 0)
            continue
        k = kc[b * capacity:b * capacity + n]
        v = vc[b * capacity:b * capacity + n]
        ref = checker.gqa_attention_f64(q[b:b + 1], k, v, [n - 1], scale)[0]
        assert checker.rel_err_normwise(got[b], ref) <= NORMWISE, b
        assert checker.rel_err_elementwise(got[b], ref) <= ELEMENTWISE, b
    return got


@pytest.mark.parametrize("length", [1, 7, 128, 129, 1000, 4096, 8192])
def test_decode_llama_1b_heads(ctx, length):
    """32 query / 8 KV heads, head_dim 64, one sequence."""
    _decode_case(ctx, 1, 32, 8, 64, [length], max(length, 1), seed=length)


@pytest.mark.parametrize("length", [1, 300, 5000])
def test_decode_head_dim_128(ctx, length):
    _decode_case(ctx, 1, 32, 8, 128, [length], length, seed=7 + length)


def test_decode_batch_of_ragged_sequences(ctx):
    """Different lengths per sequence, one of them empty, and a max_len that
    clips a sequence whose seq_len is larger."""
    lens = [513, 0, 1, 2048, 77, 3000]
    got = _decode_case(ctx, 6, 32, 8, 64, lens, 3072, seed=11, max_len=2500)
    assert got.shape == (6, 32, 64)


@pytest.mark.parametrize("qh,kvh,hd", [(8, 8, 64), (64, 8, 64), (16, 4, 128), (12, 2, 64),
                                       (32, 2, 64), (64, 2, 128), (48, 1, 64)])
def test_decode_group_sizes(ctx, qh, kvh, hd):
    _decode_case(ctx, 2, qh, kvh, hd, [700, 1900], 2048, seed=qh * 10 + kvh)


def test_decode_long_context(ctx):
    """32768 cached positions: many chunks per sequence, each warp many tiles."""
    _decode_case(ctx, 1, 32, 8, 64, [32768], 32768, seed=21)


def test_decode_repeat_is_deterministic(ctx):
    a = _decode_case(ctx, 1, 32, 8, 64, [6000], 6000, seed=5)
    b = _decode_case(ctx, 1, 32, 8, 64, [6000], 6000, seed=5)
    assert np.array_equal(a, b)


def test_decode_argument_checks(ctx):
    q = ctx.empty(plain((1, 32, 64), DType.F16))
    kc = ctx.empty(plain((128, 8, 64), DType.F16))
    lens = ctx.from_bytes(plain((1,), DType.I32), np.array([4], np.int32))
    out = ctx.empty(plain((1, 32, 64), DType.F16))
    with pytest.raises(errors.ShapeMismatch):
        ops.gqa_attention_decode_f16(ctx, q, kc, kc, lens, out, 256, 100)
    bad = ctx.empty(plain((1, 32, 96), DType.F16))
    kc96 = ctx.empty(plain((128, 8, 96), DType.F16))
    with pytest.raises(errors.Runtime):
        ops.gqa_attention_decode_f16(ctx, bad, kc96, kc96, lens, ctx.empty(
            plain((1, 32, 96), DType.F16)), 128, 100)


def _prefill_case(ctx, tokens, start, qh, kvh, seed, row0=0, extra_rows=0):
    hd = 64
    rng = np.random.default_rng(seed)
    rows = row0 + start + tokens + extra_rows
    kc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    vc = f16(rng.normal(0, 1, (rows, kvh, hd)))
    q = f16(rng.normal(0, 1, (tokens, qh, hd)))
    tq = ctx.from_bytes(plain(q.shape, DType.F16), q)
    tk = ctx.from_bytes(plain(kc.shape, DType.F16), kc)
    tv = ctx.from_bytes(plain(vc.shape, DType.F16), vc)
    to = ctx.from_bytes(plain(q.shape, DType.F16), np.full(q.shape, np.nan, np.float16))
    ops.gqa_attention_prefill_f16(ctx, tq, tk, tv, to, start, row0)
    got = np.frombuffer(ctx.read_bytes(to), np.float16).astype(np.float32).reshape(q.shape)
    assert ctx.device_status() == 0
    n = start + tokens
    ref = checker.gqa_attention_f64(q, kc[row0:row0 + n], vc[row0:row0 + n],
                                    np.arange(start, start + tokens), 1.0 / math.sqrt(hd))
    assert not np.isnan(got).any()
    assert checker.rel_err_normwise(got, ref) <= NORMWISE
    assert checker.rel_err_elementwise(got, ref) <= PREFILL_ELEMENTWISE
    return got


@pytest.mark.parametrize("tokens", [1, 5, 128, 129, 300, 512])
def test_prefill_causal_from_position_zero(ctx, tokens):
    """Llama-3.2-1B heads (32 query, 8 KV, head_dim 64): one query tile,
    ragged tiles and several key tiles per query tile."""
    _prefill_case(ctx, tokens, 0, 32, 8, seed=tokens)


@pytest.mark.parametrize("tokens,start", [(64, 200), (128, 128), (200, 1000), (1, 777)])
def test_prefill_chunk_after_cached_prefix(ctx, tokens, start):
    """A chunk whose queries start after `start` cached positions (chunked
    prefill): the first key tiles are fully visible, the last are masked."""
    _prefill_case(ctx, tokens, start, 32, 8, seed=tokens + start)


def test_prefill_sequence_at_a_cache_offset(ctx):
    """The sequence sits at cache rows row0..; rows after its last position
    hold other data (here random) that must not leak in."""
    _prefill_case(ctx, 150, 40, 32, 8, seed=9, row0=300, extra_rows=500)


@pytest.mark.parametrize("qh,kvh", [(8, 8), (64, 8), (12, 2)])
def test_prefill_group_sizes(ctx, qh, kvh):
    _prefill_case(ctx, 260, 30, qh, kvh, seed=qh + kvh)


def test_prefill_long_chunk(ctx):
    """2048 tokens: 16 query tiles x up to 16 key tiles each."""
    _prefill_case(ctx, 2048, 0, 32, 8, seed=2048)


def test_prefill_matches_decode_for_last_token(ctx):
    """The last query of a prefill chunk attends exactly what a decode step
    at that position attends."""
    rng = np.random.default_rng(21)
    tokens, start, qh, kvh, hd = 90, 300, 32, 8, 64
    n = start + tokens
    kc = f16(rng.normal(0, 1, (n, kvh, hd)))
    vc = f16(rng.normal(0, 1, (n, kvh, hd)))
    q = f16(rng.normal(0, 1, (tokens, qh, hd)))
    tk = ctx.from_bytes(plain(kc.shape, DType.F16), kc)
    tv = ctx.from_bytes(plain(vc.shape, DType.F16), vc)
    tq = ctx.from_bytes(plain(q.shape, DType.F16), q)
    to = ctx.empty(plain(q.shape, DType.F16))
    ops.gqa_attention_prefill_f16(ctx, tq, tk, tv, to, start)
    pre = np.frombuffer(ctx.read_bytes(to), np.float16).astype(np.float32).reshape(q.shape)
    tq1 = ctx.from_bytes(plain((1, qh, hd), DType.F16), q[-1:])
    lens = ctx.from_bytes(plain((1,), DType.I32), np.array([n], np.int32))
    to1 = ctx.empty(plain((1, qh, hd), DType.F16))
    ops.gqa_attention_decode_f16(ctx, tq1, tk, tv, lens, to1, n, n)
    dec = np.frombuffer(ctx.read_bytes(to1), np.float16).astype(np.float32).reshape(1, qh, hd)
    assert checker.rel_err_normwise(pre[-1:], dec) <= 2e-3
