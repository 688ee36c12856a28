"""GPU parity of the K-quant (Q4_K, Q6_K) decode and linear.

mote-reference rejects K-quants (crates/mote-reference/src/quantized.rs:152-157),
so the oracle is ggml's published dequantization restated in C
(oracle/mote_oracle.c, pinned bit for bit by gguf 0.19.0 golden vectors,
tests/test_oracle_kquants.py):
* the device decode (mote_cuda_kquant_dequantize_f32) must equal the golden
  values and the oracle bit for bit;
* the linear is held to 1e-3 normwise and element-wise (rms floor) against a
  float64 accumulation of the exactly decoded weights, as the Q4_0 decode
  path.  The Q4_K tensor-core kernel (1-16 tokens per launch, K % 256 == 0,
  16-byte aligned pointers), its split-K groups, ragged N, chunked launches
  beyond 16 tokens, the tcgen05 prefill path (more than 16 tokens, N % 16 ==
  0, and K % 2048 == 0 for Q6_K; element-wise 2e-3), the f32 output, the Q6_K tensor-core kernel (K % 2048
  == 0) and the warp-per-row kernel (unaligned input, other K) are covered.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import ops  # noqa: E402
from mote_b200._native import lib  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, QuantFormat, plain, quantized  # noqa: E402

BOUND = 1e-3
GOLDEN = np.load(Path(__file__).parent / "golden" / "kquant_golden.npz")
FMT = {"q4_k": (QuantFormat.Q4_K, 144, 2), "q6_k": (QuantFormat.Q6_K, 210, 3)}


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def kquant_weights(name: str, n: int, k: int, seed: int) -> np.ndarray:
    """Seeded super-blocks with the scale ranges of real weights
    (Q4_K: d, dmin ~ U(2e-5, 1e-4); Q6_K: d ~ U(1e-4, 6e-4)); all other
    bytes uniform."""
    rng = np.random.default_rng(seed)
    fmt, bb, _ = FMT[name]
    nb = n * (k // 256)
    b = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
    if name == "q4_k":
        b[:, 0:2] = rng.uniform(2e-5, 1e-4, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        b[:, 2:4] = rng.uniform(2e-5, 1e-4, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    else:
        b[:, 208:210] = rng.uniform(1e-4, 6e-4, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def device_decode(ctx, name, w, n, k):
    fmt, _, _ = FMT[name]
    wt = ctx.from_bytes(quantized((n, k), fmt), w)
    out = ctx.empty(plain((n, k), DType.F32))
    ops.kquant_decode_f32(ctx, wt, out)
    return np.frombuffer(ctx.read_bytes(out), np.float32).reshape(n, k)


@pytest.mark.parametrize("name", sorted(FMT))
def test_device_decode_matches_gguf_golden_bit_for_bit(ctx, name):
    blocks = GOLDEN[f"{name}_blocks"]
    got = device_decode(ctx, name, blocks.reshape(-1), 1, blocks.shape[0] * 256)
    assert got.view(np.uint32).reshape(-1).tolist() == GOLDEN[f"{name}_values"].tolist()
    assert ctx.device_status() == 0


@pytest.mark.parametrize("name", sorted(FMT))
def test_device_decode_matches_oracle(ctx, oracle_lib, name):
    n, k = 37, 1280
    w = kquant_weights(name, n, k, seed=11)
    fmt_id = FMT[name][2]
    want = oracle_lib.kquant_dequantize(w, fmt_id, n, k)
    got = device_decode(ctx, name, w, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def run(ctx, name, x, w, m, n, k, out_dtype=DType.F16):
    fmt, _, _ = FMT[name]
    xt = ctx.from_bytes(plain((m, k), DType.F16), x.astype(np.float16))
    wt = ctx.from_bytes(quantized((n, k), fmt), w)
    yt = ctx.empty(plain((m, n), out_dtype))
    ops.quantized_linear_kquant(ctx, xt, wt, yt, out_dtype)
    np_out = np.float16 if out_dtype is DType.F16 else np.float32
    got = np.frombuffer(ctx.read_bytes(yt), np_out).astype(np.float32).reshape(m, n)
    assert ctx.device_status() == 0
    return got


def tensor_core_path(name, m, n, k):
    """More than 16 tokens with N % 16 == 0 and K % 256 == 0 (Q4_K) or
    K % 2048 == 0 (Q6_K) run on the tcgen05 GEMM, which rounds each weight's
    f32 value to f16 once (<= 2^-11 relative): element-wise bound 2e-3
    there, as for the Q4_0 and Q8_0 prefill paths."""
    return m > 16 and n % 16 == 0 and k % (256 if name == "q4_k" else 2048) == 0


def check(oracle_lib, name, got, x, w, m, n, k):
    x32 = x.astype(np.float16).astype(np.float32)
    ref64 = oracle_lib.kquant_linear_f64(x32, w, FMT[name][2], m, n, k)
    assert checker.rel_err_normwise(got, ref64) <= BOUND
    elementwise = 2e-3 if tensor_core_path(name, m, n, k) else BOUND
    assert checker.rel_err_elementwise(got, ref64) <= elementwise


@pytest.mark.parametrize("m,n,k", [(17, 256, 256), (64, 4096, 4096), (200, 528, 1024),
                                   (129, 16, 768), (300, 2048, 2048), (40, 2048, 2048)])
def test_q4_k_prefill_tensor_cores(ctx, oracle_lib, m, n, k):
    """More than 16 tokens on the tcgen05 GEMM with the Q4_K converter (one
    144-byte super-block per raw row, each value (d*sc)*q - dmin*m in f32
    rounded once to f16); ragged M."""
    w = kquant_weights("q4_k", n, k, seed=60 + m)
    x = np.random.default_rng(61 + m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, "q4_k", run(ctx, "q4_k", x, w, m, n, k), x, w, m, n, k)


@pytest.mark.parametrize("m,n,k", [(17, 256, 2048), (64, 4096, 4096), (200, 528, 2048),
                                   (129, 16, 6144), (300, 2048, 2048), (40, 96, 16384)])
def test_q6_k_prefill_tensor_cores(ctx, oracle_lib, m, n, k):
    """More than 16 tokens with K % 2048 == 0 on the tcgen05 GEMM with the Q6_K
    converter (240-byte TMA windows, each value (d*sc)*(q-32) in f32 rounded
    once to f16); ragged M, every window offset."""
    w = kquant_weights("q6_k", n, k, seed=80 + m)
    x = np.random.default_rng(81 + m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, "q6_k", run(ctx, "q6_k", x, w, m, n, k), x, w, m, n, k)


def test_q4_k_prefill_full_size_sampled(ctx, oracle_lib):
    """M=2048, K=4096, N=14336 on the tensor cores; 64 sampled rows x all N
    against float64 over the oracle's decoded weights."""
    m, n, k = 2048, 14336, 4096
    w = kquant_weights("q4_k", n, k, seed=77)
    x = np.random.default_rng(78).normal(0, 1, (m, k)).astype(np.float16)
    got = run(ctx, "q4_k", x, w, m, n, k)
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    dec = oracle_lib.kquant_dequantize(w, FMT["q4_k"][2], n, k).astype(np.float64)
    ref64 = x[rows].astype(np.float64) @ dec.T
    assert checker.rel_err_normwise(got[rows], ref64) <= BOUND
    assert checker.rel_err_elementwise(got[rows], ref64) <= 2e-3


@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16, 17, 40])
@pytest.mark.parametrize("n,k", [(2048, 2048), (40, 256), (300, 4096)])
def test_q4_k_linear_matches_oracle(ctx, oracle_lib, m, n, k):
    w = kquant_weights("q4_k", n, k, seed=n + k)
    x = np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, "q4_k", run(ctx, "q4_k", x, w, m, n, k), x, w, m, n, k)


@pytest.mark.parametrize("m,n,k", [(1, 1000, 8192), (4, 528, 14336), (16, 64, 6144),
                                   (1, 16032, 4096), (12, 4096, 4096)])
def test_q4_k_long_k_and_splits(ctx, oracle_lib, m, n, k):
    w = kquant_weights("q4_k", n, k, seed=7 + n)
    x = np.random.default_rng(9 + m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, "q4_k", run(ctx, "q4_k", x, w, m, n, k), x, w, m, n, k)


@pytest.mark.parametrize("m", [1, 16])
def test_q4_k_f32_output(ctx, oracle_lib, m):
    n, k = 300, 2048
    w = kquant_weights("q4_k", n, k, seed=21)
    x = np.random.default_rng(22).normal(0, 1, (m, k)).astype(np.float16)
    got = run(ctx, "q4_k", x, w, m, n, k, DType.F32)
    check(oracle_lib, "q4_k", got, x, w, m, n, k)
    # f32 out is the unrounded accumulator of the same kernel
    f16 = run(ctx, "q4_k", x, w, m, n, k)
    assert np.array_equal(got.astype(np.float16).astype(np.float32), f16)


def test_q4_k_unaligned_input_runs_the_generic_kernel(ctx, oracle_lib):
    """An input 2 bytes past a 16-byte boundary takes the warp-per-row
    kernel (through the C ABI: the ops layer accepts only offset-0 tensors)."""
    m, n, k = 3, 70, 512
    w = kquant_weights("q4_k", n, k, seed=5)
    x = np.random.default_rng(6).normal(0, 1, (m, k)).astype(np.float16)
    buf = ctx.empty(plain((m * k + 8,), DType.F16))
    raw = np.zeros(m * k + 8, np.float16)
    raw[1:1 + m * k] = x.reshape(-1)
    ctx.upload_numpy(buf, raw)
    wt = ctx.from_bytes(quantized((n, k), QuantFormat.Q4_K), w)
    yt = ctx.empty(plain((m, n), DType.F16))
    st = lib().mote_cuda_quantized_linear_q4_k_f16(buf.pointer + 2, wt.pointer, yt.pointer, m,
                                                    n, k, ctx.stream)
    assert st == 0
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n)
    check(oracle_lib, "q4_k", got, x, w, m, n, k)


@pytest.mark.parametrize("m,n,k", [(1, 2048, 2048), (5, 300, 4096), (17, 40, 256),
                                   (1, 1000, 8192), (16, 100, 6144), (9, 2048, 4096),
                                   (3, 50, 2304), (12, 4096, 2048), (2, 16032, 4096)])
def test_q6_k_linear_matches_oracle(ctx, oracle_lib, m, n, k):
    """K % 2048 == 0 with aligned pointers: the tensor-core Q6_K kernel (odd
    super-blocks 2 bytes off a word); other K: the warp-per-row kernel."""
    w = kquant_weights("q6_k", n, k, seed=3 * n + k)
    x = np.random.default_rng(m + 100).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, "q6_k", run(ctx, "q6_k", x, w, m, n, k), x, w, m, n, k)


def test_kquant_linear_rejects_misaligned_k(ctx):
    f = lib().mote_cuda_quantized_linear_q4_k_f16
    assert f(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 16, 288,
             ctx.stream) == 1


def test_gguf_weights_load_and_run(ctx, oracle_lib, tmp_path):
    """A GGUF file (written by the gguf package) mapped by mote_b200.gguf_file,
    its Q4_K, Q6_K and Q4_0 tensors copied to the device and run through the
    linears; results against the oracle on the same bytes."""
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T

    from mote_b200.gguf_file import GGUFFile, load_tensors

    n, k, m = 96, 1024, 3
    w4k = kquant_weights("q4_k", n, k, seed=31).reshape(n, -1)
    w6k = kquant_weights("q6_k", n, k, seed=32).reshape(n, -1)
    w40 = np.empty((n, k // 32, 18), np.uint8)
    rng = np.random.default_rng(33)
    w40[:, :, 0:2] = rng.uniform(1e-3, 3e-3, (n, k // 32)).astype(np.float16).view(
        np.uint8).reshape(n, k // 32, 2)
    w40[:, :, 2:] = rng.integers(0, 256, (n, k // 32, 16), dtype=np.uint8)
    w40 = w40.reshape(n, -1)
    path = tmp_path / "w.gguf"
    wr = gguf.GGUFWriter(str(path), "llama")
    wr.add_tensor("blk.0.ffn_up.weight", w4k, raw_dtype=T.Q4_K)
    wr.add_tensor("blk.0.ffn_down.weight", w6k, raw_dtype=T.Q6_K)
    wr.add_tensor("blk.0.attn_q.weight", w40, raw_dtype=T.Q4_0)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    x = np.random.default_rng(34).normal(0, 1, (m, k)).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    with GGUFFile(path) as f:
        dev = load_tensors(ctx, f)
    for name, fmt_name, raw in (("blk.0.ffn_up.weight", "q4_k", w4k),
                                ("blk.0.ffn_down.weight", "q6_k", w6k)):
        yt = ctx.empty(plain((m, n), DType.F16))
        ops.quantized_linear_kquant(ctx, xt, dev[name], yt)
        got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n)
        check(oracle_lib, fmt_name, got, x, raw.reshape(-1), m, n, k)
    yt = ctx.empty(plain((m, n), DType.F16))
    ops.quantized_linear_q4_0_f16(ctx, xt, dev["blk.0.attn_q.weight"], yt)
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n)
    ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w40.reshape(-1), n, k))
    assert checker.rel_err_normwise(got, ref64) <= BOUND
    assert ctx.device_status() == 0
