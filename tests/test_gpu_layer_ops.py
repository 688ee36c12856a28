"""GPU parity of the per-token layer kernels against the CPU oracle.

Mirrors crates/mote-backend-hip/tests/{rms_norm,fused_add_rms_norm,rope}.rs:
f16-quantized formula inputs, the f32 oracle's output rounded to f16, and
the reference tolerance abs 3e-3 / rel 3e-3; plus the bound of the
specification (element-wise relative error against float64 <= 1e-3 with an
rms floor) and bit-exactness where the arithmetic allows it: RoPE uses the
oracle's exact f32 operation order, so its f16 outputs must equal the
f16-rounded oracle bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker
from tests import _fixtures as fx

pytestmark = pytest.mark.gpu

from mote_b200 import errors, ops  # noqa: E402
from mote_b200.context import CudaContext, Tensor  # noqa: E402
from mote_b200.types import DType, RopeLayout, plain  # noqa: E402

EPS = 1e-6


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def up16(ctx, values, shape):
    return ctx.from_bytes(plain(shape, DType.F16), fx.f16(values).reshape(-1))


def up32(ctx, values, shape):
    return ctx.from_bytes(plain(shape, DType.F32), np.asarray(values, np.float32).reshape(-1))


def read16(ctx, t):
    return np.frombuffer(ctx.read_bytes(t), np.float16).astype(np.float32)


# ---- RMSNorm -----------------------------------------------------------------
@pytest.mark.parametrize("rows,hidden", [(3, 513), (512, 2048), (4, 4096), (2, 8192),
                                         (5, 16384), (1, 8)])
def test_rms_norm_matches_oracle(ctx, oracle_lib, rows, hidden):
    x = fx.f16(fx.norm_input(rows * hidden))
    w = fx.f16(fx.norm_weight(hidden))
    xt, wt = up16(ctx, x, (rows, hidden)), up16(ctx, w, (hidden,))
    out = ctx.empty(plain((rows, hidden), DType.F16))
    ops.rms_norm_f16(ctx, xt, wt, out, EPS)
    got = read16(ctx, out)
    want = checker.f16_round(oracle_lib.rms_norm_f32(x.astype(np.float32),
                                                     w.astype(np.float32), hidden, EPS))
    ok, bad = checker.within_reference_tolerance(got, want, 3e-3, 3e-3)
    assert ok, bad
    ref64 = checker.rms_norm_f64(x, w, hidden, EPS)
    assert checker.rel_err_elementwise(got, ref64) <= 1e-3


def test_rms_norm_in_place(ctx, oracle_lib):
    rows, hidden = 3, 2048
    x = fx.f16(fx.norm_input(rows * hidden))
    w = fx.f16(fx.norm_weight(hidden))
    xt, wt = up16(ctx, x, (rows, hidden)), up16(ctx, w, (hidden,))
    ops.rms_norm_f16(ctx, xt, wt, xt, EPS)
    want = checker.f16_round(oracle_lib.rms_norm_f32(x.astype(np.float32),
                                                     w.astype(np.float32), hidden, EPS))
    ok, bad = checker.within_reference_tolerance(read16(ctx, xt), want, 3e-3, 3e-3)
    assert ok, bad


def test_rms_norm_empty_and_validation(ctx):
    """rms_norm.rs:64-142: empty tensors, epsilon, shapes, foreign storage."""
    w = up16(ctx, np.ones(513), (513,))
    ops.rms_norm_f16(ctx, ctx.empty(plain((0, 513), DType.F16)), w,
                     ctx.empty(plain((0, 513), DType.F16)), EPS)
    ops.rms_norm_f16(ctx, ctx.empty(plain((2, 0), DType.F16)), ctx.empty(plain((0,), DType.F16)),
                     ctx.empty(plain((2, 0), DType.F16)), EPS)
    x = up16(ctx, fx.norm_input(3 * 513), (3, 513))
    out = ctx.empty(plain((3, 513), DType.F16))
    for eps in (-EPS, float("nan"), float("inf"), float("-inf")):
        with pytest.raises(errors.InvalidEpsilon):
            ops.rms_norm_f16(ctx, x, w, out, eps)
    with pytest.raises(errors.ShapeMismatch) as e:
        ops.rms_norm_f16(ctx, x, w, ctx.empty(plain((3, 514), DType.F16)), EPS)
    assert e.value.tensor == "output"
    with pytest.raises(errors.ShapeMismatch) as e:
        ops.rms_norm_f16(ctx, x, ctx.empty(plain((512,), DType.F16)), out, EPS)
    assert e.value.tensor == "weight"
    with pytest.raises(errors.WrongStorage):
        ops.rms_norm_f16(ctx, x, w, CudaContext(0).empty(plain((3, 513), DType.F16)), EPS)
    with pytest.raises(errors.DTypeMismatch):
        ops.rms_norm_f16(ctx, x, w, ctx.empty(plain((3, 513), DType.F32)), EPS)


# ---- fused add + RMSNorm -----------------------------------------------------------
def _fused_expect(oracle_lib, x, r, w, hidden):
    norm, res = oracle_lib.fused_add_rms_norm_f32(x.astype(np.float32), r.astype(np.float32),
                                                  w.astype(np.float32), hidden, EPS)
    return checker.f16_round(norm), checker.f16_round(res)


@pytest.mark.parametrize("rows,hidden", [(3, 513), (1, 2048), (64, 2048), (2, 8192)])
def test_fused_add_rms_norm_matches_oracle(ctx, oracle_lib, rows, hidden):
    x = fx.f16(fx.norm_input(rows * hidden))
    r = fx.f16(fx.residual_input(rows * hidden))
    w = fx.f16(fx.norm_weight(hidden))
    xt, rt, wt = up16(ctx, x, (rows, hidden)), up16(ctx, r, (rows, hidden)), up16(ctx, w, (hidden,))
    out = ctx.empty(plain((rows, hidden), DType.F16))
    ops.fused_add_rms_norm_f16(ctx, xt, rt, wt, out, EPS)
    want_n, want_r = _fused_expect(oracle_lib, x, r, w, hidden)
    for got, want in ((read16(ctx, out), want_n), (read16(ctx, rt), want_r)):
        ok, bad = checker.within_reference_tolerance(got, want, 3e-3, 3e-3)
        assert ok, bad
    # the residual sum is a single f32 add rounded to f16: bit-exact
    assert np.array_equal(read16(ctx, rt), want_r)


def test_fused_in_place_and_input_aliasing_residual(ctx, oracle_lib):
    """fused_add_rms_norm.rs:81-152."""
    rows, hidden = 3, 513
    x = fx.f16(fx.norm_input(rows * hidden))
    r = fx.f16(fx.residual_input(rows * hidden))
    w = fx.f16(fx.norm_weight(hidden))
    xt, rt, wt = up16(ctx, x, (rows, hidden)), up16(ctx, r, (rows, hidden)), up16(ctx, w, (hidden,))
    ops.fused_add_rms_norm_f16(ctx, xt, rt, wt, xt, EPS)  # output aliases input
    want_n, want_r = _fused_expect(oracle_lib, x, r, w, hidden)
    assert checker.within_reference_tolerance(read16(ctx, xt), want_n, 3e-3, 3e-3)[0]
    assert np.array_equal(read16(ctx, rt), want_r)
    xt = up16(ctx, x, (rows, hidden))
    out = ctx.empty(plain((rows, hidden), DType.F16))
    ops.fused_add_rms_norm_f16(ctx, xt, xt, wt, out, EPS)  # residual aliases input
    want_n, want_r = _fused_expect(oracle_lib, x, x, w, hidden)
    assert checker.within_reference_tolerance(read16(ctx, out), want_n, 3e-3, 3e-3)[0]
    assert np.array_equal(read16(ctx, xt), want_r)


def test_fused_aliasing_rules(ctx):
    """fused_add_rms_norm.rs:154-249."""
    rows, hidden = 3, 513
    xt = up16(ctx, fx.norm_input(rows * hidden), (rows, hidden))
    rt = up16(ctx, fx.residual_input(rows * hidden), (rows, hidden))
    wt = up16(ctx, fx.norm_weight(hidden), (hidden,))
    out = ctx.empty(plain((rows, hidden), DType.F16))
    with pytest.raises(errors.AliasedStorage) as e:
        ops.fused_add_rms_norm_f16(ctx, xt, rt, wt, rt, EPS)
    assert (e.value.tensor, e.value.other) == ("output", "residual")
    w_on_out = Tensor(plain((hidden,), DType.F16), out.storage, 0)
    with pytest.raises(errors.AliasedStorage) as e:
        ops.fused_add_rms_norm_f16(ctx, xt, rt, w_on_out, out, EPS)
    assert (e.value.tensor, e.value.other) == ("weight", "output")
    w_on_res = Tensor(plain((hidden,), DType.F16), rt.storage, 0)
    with pytest.raises(errors.AliasedStorage) as e:
        ops.fused_add_rms_norm_f16(ctx, xt, rt, w_on_res, out, EPS)
    assert (e.value.tensor, e.value.other) == ("weight", "residual")
    with pytest.raises(errors.ShapeMismatch) as e:
        ops.fused_add_rms_norm_f16(ctx, xt, ctx.empty(plain((rows + 1, hidden), DType.F16)), wt,
                                   out, EPS)
    assert e.value.tensor == "residual"


# ---- RoPE --------------------------------------------------------------------------
def _rope_case(ctx, oracle_lib, leading, heads, head_dim, rot, layout, in_place):
    shape = tuple(leading) + (heads, head_dim)
    cache = tuple(leading) + (rot // 2,)
    n = int(np.prod(shape))
    nc = int(np.prod(cache))
    tokens = int(np.prod(leading)) if leading else 1
    x = fx.f16(fx.norm_input(n))
    c, s = fx.rope_cos(nc), fx.rope_sin(nc)
    xt = up16(ctx, x, shape)
    ct, st = up32(ctx, c, cache), up32(ctx, s, cache)
    out = xt if in_place else ctx.empty(plain(shape, DType.F16))
    ops.rope_f16(ctx, xt, ct, st, out, rot, layout)
    got = np.frombuffer(ctx.read_bytes(out), np.float16)
    want = oracle_lib.rope_f32(x.astype(np.float32), c, s, tokens, heads, head_dim, rot,
                               layout.value).astype(np.float16)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    tail = (np.arange(n) % head_dim) >= rot
    assert np.array_equal(got.view(np.uint16)[tail], x.view(np.uint16)[tail])


@pytest.mark.parametrize("layout", [RopeLayout.HalfSplit, RopeLayout.Interleaved])
@pytest.mark.parametrize("leading", [(2,), (), (2, 2)])
@pytest.mark.parametrize("in_place", [False, True])
def test_rope_matches_oracle_bit_exact(ctx, oracle_lib, layout, leading, in_place):
    """rope.rs:25-51,340-431: [tokens, 3, 70], rotary_dim 66, both layouts."""
    _rope_case(ctx, oracle_lib, leading, 3, 70, 66, layout, in_place)


def test_rope_llama_shapes(ctx, oracle_lib):
    _rope_case(ctx, oracle_lib, (512,), 32, 64, 64, RopeLayout.HalfSplit, False)
    _rope_case(ctx, oracle_lib, (7,), 8, 128, 128, RopeLayout.Interleaved, True)
    _rope_case(ctx, oracle_lib, (1,), 2, 6, 0, RopeLayout.HalfSplit, False)


def test_rope_empty_and_validation(ctx):
    """rope.rs:53-330 (empty tensors, rotary dim, cache shapes)."""
    cache = up32(ctx, np.zeros(2 * 33), (2, 33))
    ops.rope_f16(ctx, ctx.empty(plain((0, 3, 70), DType.F16)),
                 ctx.empty(plain((0, 33), DType.F32)), ctx.empty(plain((0, 33), DType.F32)),
                 ctx.empty(plain((0, 3, 70), DType.F16)), 66, RopeLayout.HalfSplit)
    ops.rope_f16(ctx, ctx.empty(plain((2, 0, 70), DType.F16)), cache, cache,
                 ctx.empty(plain((2, 0, 70), DType.F16)), 66, RopeLayout.HalfSplit)
    x = up16(ctx, fx.norm_input(2 * 3 * 70), (2, 3, 70))
    out = ctx.empty(plain((2, 3, 70), DType.F16))
    for rot in (65, 72):
        with pytest.raises(errors.InvalidRotaryDim):
            ops.rope_f16(ctx, x, cache, cache, out, rot, RopeLayout.HalfSplit)
    with pytest.raises(errors.ShapeMismatch) as e:
        ops.rope_f16(ctx, x, up32(ctx, np.zeros(2 * 32), (2, 32)), cache, out, 66,
                     RopeLayout.HalfSplit)
    assert e.value.tensor == "cos"
    with pytest.raises(errors.RankTooSmall):
        ops.rope_f16(ctx, up16(ctx, np.zeros(70), (70,)), cache, cache, out, 66,
                     RopeLayout.HalfSplit)


# ---- fused RMSNorm + RoPE (config 2) ---------------------------------------------
@pytest.mark.parametrize("layout", [RopeLayout.HalfSplit, RopeLayout.Interleaved])
@pytest.mark.parametrize("tokens,hidden,qh,kh,hd", [(512, 2048, 32, 8, 64), (5, 4096, 32, 8, 128),
                                                  (3, 520, 2, 1, 64), (2, 96, 3, 1, 30)])
def test_rms_norm_rope_fused(ctx, oracle_lib, layout, tokens, hidden, qh, kh, hd):
    rng = np.random.default_rng(tokens + hidden)
    x = fx.f16(rng.normal(0, 1, tokens * hidden))
    gamma = fx.f16(1.0 + rng.normal(0, 0.1, hidden))
    q = fx.f16(rng.normal(0, 1, tokens * qh * hd))
    k = fx.f16(rng.normal(0, 1, tokens * kh * hd))
    pos = np.arange(tokens, dtype=np.int32)
    cos, sin = oracle_lib.rope_cos_sin_f64(pos, hd, 10000.0)
    xt, gt = up16(ctx, x, (tokens, hidden)), up16(ctx, gamma, (hidden,))
    qt, kt = up16(ctx, q, (tokens, qh, hd)), up16(ctx, k, (tokens, kh, hd))
    ct, st = up32(ctx, cos, (tokens, hd // 2)), up32(ctx, sin, (tokens, hd // 2))
    xo = ctx.empty(plain((tokens, hidden), DType.F16))
    qo = ctx.empty(plain((tokens, qh, hd), DType.F16))
    ko = ctx.empty(plain((tokens, kh, hd), DType.F16))
    ops.rms_norm_rope_f16(ctx, xt, gt, xo, qt, qo, kt, ko, ct, st, EPS, layout)
    want_x = checker.f16_round(oracle_lib.rms_norm_f32(x.astype(np.float32),
                                                       gamma.astype(np.float32), hidden, EPS))
    got_x = read16(ctx, xo)
    assert checker.within_reference_tolerance(got_x, want_x, 3e-3, 3e-3)[0]
    assert checker.rel_err_elementwise(got_x, checker.rms_norm_f64(x, gamma, hidden, EPS)) <= 1e-3
    for src, dst, heads in ((q, qo, qh), (k, ko, kh)):
        want = oracle_lib.rope_f32(src.astype(np.float32), cos, sin, tokens, heads, hd, hd,
                                   layout.value).astype(np.float16)
        got = np.frombuffer(ctx.read_bytes(dst), np.float16)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
        ref64 = checker.rope_f64(src, cos, sin, tokens, heads, hd, hd, layout.value)
        assert checker.rel_err_elementwise(got, ref64) <= 1e-3


# ---- SwiGLU, embedding gather, cos/sin table ----------------------------------------
@pytest.mark.parametrize("n", [8192, 8193, 3])
def test_swiglu(ctx, n):
    rng = np.random.default_rng(n)
    g, u = fx.f16(rng.normal(0, 2, n)), fx.f16(rng.normal(0, 1, n))
    gt, ut = up16(ctx, g, (n,)), up16(ctx, u, (n,))
    out = ctx.empty(plain((n,), DType.F16))
    ops.swiglu_f16(ctx, gt, ut, out)
    ref = checker.swiglu_f64(g, u)
    got = read16(ctx, out)
    assert checker.rel_err_elementwise(got, ref) <= 1e-3
    assert np.all(np.abs(got - ref) <= np.maximum(1e-3, 1e-3 * np.abs(ref)))


def test_embedding_gather_bit_exact(ctx, oracle_lib):
    vocab, hidden, tokens = 128256, 2048, 64
    rng = np.random.default_rng(9)
    table = fx.f16(rng.normal(0, 0.02, (vocab, hidden)))
    ids = rng.integers(0, vocab, tokens).astype(np.int32)
    ids[0], ids[1] = 0, vocab - 1
    tt = ctx.from_bytes(plain((vocab, hidden), DType.F16), table)
    it = ctx.from_bytes(plain((tokens,), DType.I32), ids)
    out = ctx.empty(plain((tokens, hidden), DType.F16))
    ops.embedding_gather_f16(ctx, tt, it, out)
    want, flag = oracle_lib.embedding_gather_f16(table.view(np.uint16), vocab, hidden, ids)
    assert flag == 0
    assert np.array_equal(np.frombuffer(ctx.read_bytes(out), np.uint16), want)


def test_embedding_gather_out_of_range_ids(ctx, oracle_lib):
    vocab, hidden = 10, 24  # hidden*2 = 48 bytes: vector path
    table = fx.f16(np.arange(vocab * hidden, dtype=np.float32) / 64)
    ids = np.array([3, -1, 10, 9], np.int32)
    tt = ctx.from_bytes(plain((vocab, hidden), DType.F16), table)
    it = ctx.from_bytes(plain((4,), DType.I32), ids)
    out = ctx.empty(plain((4, hidden), DType.F16))
    with pytest.raises(errors.IndexOutOfRange):
        ops.embedding_gather_f16(ctx, tt, it, out)
    want, flag = oracle_lib.embedding_gather_f16(table.view(np.uint16), vocab, hidden, ids)
    assert flag == 1
    assert np.array_equal(np.frombuffer(ctx.read_bytes(out), np.uint16), want)
    # odd hidden: scalar path
    t2 = ctx.from_bytes(plain((vocab, 5), DType.F16), table[: vocab * 5])
    o2 = ctx.empty(plain((4, 5), DType.F16))
    with pytest.raises(errors.IndexOutOfRange):
        ops.embedding_gather_f16(ctx, t2, it, o2)
    want2, _ = oracle_lib.embedding_gather_f16(table[: vocab * 5].view(np.uint16), vocab, 5, ids)
    assert np.array_equal(np.frombuffer(ctx.read_bytes(o2), np.uint16), want2)


def test_rope_cos_sin_table(ctx, oracle_lib):
    tokens, rot = 512, 64
    pos = np.arange(tokens, dtype=np.int32)
    pt = ctx.from_bytes(plain((tokens,), DType.I32), pos)
    ct = ctx.empty(plain((tokens, rot // 2), DType.F32))
    st = ctx.empty(plain((tokens, rot // 2), DType.F32))
    ops.rope_cos_sin_f32(ctx, pt, ct, st, 10000.0)
    want_c, want_s = oracle_lib.rope_cos_sin_f64(pos, rot, 10000.0)
    got_c = np.frombuffer(ctx.read_bytes(ct), np.float32).reshape(tokens, rot // 2)
    got_s = np.frombuffer(ctx.read_bytes(st), np.float32).reshape(tokens, rot // 2)
    # f64 evaluation rounded once to f32 on both sides: at most 1 ulp apart
    assert checker.ulp_distance_f32(got_c, want_c).max() <= 1
    assert checker.ulp_distance_f32(got_s, want_s).max() <= 1
