"""C ABI checks that need no GPU.

* the library loads and exports every function ``include/mote_cuda.h``
  declares, and the Python binding declares the same set;
* every launcher rejects invalid arguments with the reference shim's status
  code before touching the device, and returns 0 for validated empty sizes
  (these paths never reach the CUDA runtime, so they run on CPU hosts).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from mote_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "mote_cuda.h"
FAKE = 0x1000  # never dereferenced: every call below returns before launching
STREAM = 0x2000


def declared_symbols() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(mote_cuda_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    return _native.lib()


def test_library_exports_every_declared_symbol(lib):
    symbols = declared_symbols()
    assert len(symbols) >= 30
    for name in sorted(symbols):
        assert hasattr(lib, name), name


def test_python_binding_matches_header():
    assert declared_symbols() == set(_native.SIGNATURES)


def test_abi_version(lib):
    assert lib.mote_cuda_abi_version() == 1


LINEARS = ["mote_cuda_quantized_linear_q4_0_f16", "mote_cuda_quantized_linear_q4_0_f16_f32out",
           "mote_cuda_quantized_linear_q4_0_f32"]


@pytest.mark.parametrize("name", LINEARS)
def test_linear_argument_rules(lib, name):
    fn = getattr(lib, name)
    # quantized_linear.hip:64-76: null pointers, stream included -> 1
    assert fn(None, FAKE, FAKE, 1, 1, 32, STREAM) == 1
    assert fn(FAKE, None, FAKE, 1, 1, 32, STREAM) == 1
    assert fn(FAKE, FAKE, None, 1, 1, 32, STREAM) == 1
    assert fn(FAKE, FAKE, FAKE, 1, 1, 32, None) == 1
    # K not a multiple of 32 -> 1
    assert fn(FAKE, FAKE, FAKE, 1, 1, 33, STREAM) == 1
    # empty outputs -> 0 without a launch
    assert fn(FAKE, FAKE, FAKE, 0, 5, 64, STREAM) == 0
    assert fn(FAKE, FAKE, FAKE, 3, 0, 64, STREAM) == 0
    # rows * N beyond 32 bits -> 9 (cudaErrorInvalidConfiguration)
    assert fn(FAKE, FAKE, FAKE, 1 << 32, 1, 32, STREAM) == 9
    assert fn(FAKE, FAKE, FAKE, 1 << 17, 1 << 17, 32, STREAM) == 9


def test_gate_up_argument_rules(lib):
    fn = lib.mote_cuda_q4_0_gate_up_swiglu_f16
    assert fn(FAKE, FAKE, None, FAKE, 1, 8, 32, STREAM) == 1
    assert fn(FAKE, FAKE, FAKE, FAKE, 1, 8, 33, STREAM) == 1
    assert fn(FAKE, FAKE, FAKE, FAKE, 0, 8, 32, STREAM) == 0


def test_rms_norm_argument_rules(lib):
    fn = lib.mote_cuda_rms_norm_f16
    eps = ctypes.c_float(1e-6)
    # rms_norm.hip:166-174
    assert fn(None, FAKE, FAKE, 1, 8, eps, STREAM) == -1
    assert fn(FAKE, FAKE, FAKE, 1, 8, eps, None) == -1
    assert fn(FAKE, FAKE, FAKE, 0, 8, eps, STREAM) == 0
    assert fn(FAKE, FAKE, FAKE, 3, 0, eps, STREAM) == 0
    assert fn(FAKE, FAKE, FAKE, 1 << 32, 8, eps, STREAM) == -1


def test_fused_add_rms_norm_argument_rules(lib):
    fn = lib.mote_cuda_fused_add_rms_norm_f16
    # fused_add_rms_norm.hip:296-312
    assert fn(FAKE, None, FAKE, FAKE, 1, 8, ctypes.c_float(1e-6), STREAM) == -1
    for bad in (float("nan"), float("inf"), -1e-6):
        assert fn(FAKE, 0x3000, FAKE, FAKE, 1, 8, ctypes.c_float(bad), STREAM) == -1
    assert fn(FAKE, 0x3000, FAKE, 0x3000, 1, 8, ctypes.c_float(1e-6), STREAM) == -1
    assert fn(FAKE, 0x3000, FAKE, FAKE, 0, 8, ctypes.c_float(1e-6), STREAM) == 0


def test_rope_argument_rules(lib):
    fn = lib.mote_cuda_rope_f16
    # rope.hip:436-457
    assert fn(None, FAKE, FAKE, FAKE, 1, 1, 4, 4, 0, STREAM) == -1
    assert fn(FAKE, None, FAKE, FAKE, 1, 1, 4, 4, 0, STREAM) == -1
    assert fn(FAKE, FAKE, FAKE, FAKE, 1, 1, 4, 4, 2, STREAM) == -1  # unknown layout
    assert fn(FAKE, FAKE, FAKE, FAKE, 1, 1, 4, 3, 0, STREAM) == -1  # odd rotary_dim
    assert fn(FAKE, FAKE, FAKE, FAKE, 1, 1, 4, 6, 0, STREAM) == -1  # rotary_dim > head_dim
    assert fn(FAKE, FAKE, FAKE, FAKE, 0, 3, 8, 8, 0, STREAM) == 0
    assert fn(FAKE, FAKE, FAKE, FAKE, 2, 0, 8, 8, 0, STREAM) == 0
    assert fn(FAKE, FAKE, FAKE, FAKE, 1 << 31, 4, 8, 8, 0, STREAM) == -1


def test_rope_zero_rotary_dim_accepts_null_tables(lib):
    # rotary_dim == 0 is a pure copy; null tables are tolerated (rope.hip:439-444)
    # but we still must not launch here: zero tokens.
    assert lib.mote_cuda_rope_f16(FAKE, None, None, FAKE, 0, 1, 4, 0, 0, STREAM) == 0


def test_new_op_argument_rules(lib):
    assert lib.mote_cuda_swiglu_f16(None, FAKE, FAKE, 8, STREAM) == -1
    assert lib.mote_cuda_swiglu_f16(FAKE, FAKE, FAKE, 0, STREAM) == 0
    assert lib.mote_cuda_embedding_gather_f16(FAKE, FAKE, FAKE, 1, 8, 8, None, STREAM) == -1
    assert lib.mote_cuda_embedding_gather_f16(FAKE, FAKE, FAKE, 0, 8, 8, FAKE, STREAM) == 0
    assert lib.mote_cuda_q4_0_decode_f32(FAKE, FAKE, 1, 33, STREAM) == 1
    assert lib.mote_cuda_q4_0_encode_f32(FAKE + 4, FAKE, 1, 32, STREAM) == 1  # unaligned input
    assert lib.mote_cuda_rope_cos_sin_f32(FAKE, FAKE, FAKE, 1, 3, ctypes.c_double(1e4),
                                          STREAM) == -1
    eps = ctypes.c_float(1e-6)
    assert lib.mote_cuda_rms_norm_rope_f16(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE,
                                           0, 64, 1, 1, 64, 0, eps, STREAM) == 0
    assert lib.mote_cuda_rms_norm_rope_f16(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE,
                                           1, 64, 1, 1, 64, 5, eps, STREAM) == -1


def test_attention_argument_rules(lib):
    scale = ctypes.c_float(0.125)
    # KV-cache append: null pointers, empty, rows not in 16-byte vectors, alignment
    assert lib.mote_cuda_kv_cache_append_f16(None, FAKE, FAKE, FAKE, FAKE, 1, 8, 64, 16, None,
                                             STREAM) == 1
    assert lib.mote_cuda_kv_cache_append_f16(FAKE, FAKE, FAKE, FAKE, FAKE, 0, 8, 64, 16, None,
                                             STREAM) == 0
    assert lib.mote_cuda_kv_cache_append_f16(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 1, 4, 16, None,
                                             STREAM) == 1
    assert lib.mote_cuda_kv_cache_append_f16(FAKE + 8, FAKE, FAKE, FAKE, FAKE, 1, 8, 64, 16, None,
                                             STREAM) == 1
    # decode: nulls, empty batch, group, head_dim, max_len beyond the capacity, scale
    dec = lib.mote_cuda_gqa_attention_decode_f16
    assert dec(None, FAKE, FAKE, FAKE, FAKE, 1, 32, 8, 64, 64, 64, scale, None, 0, STREAM) == 1
    assert dec(FAKE, FAKE, FAKE, FAKE, FAKE, 0, 32, 8, 64, 64, 64, scale, None, 0, STREAM) == 0
    assert dec(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 30, 8, 64, 64, 64, scale, None, 0, STREAM) == 1
    assert dec(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 32, 8, 96, 64, 64, scale, None, 0, STREAM) == 1
    assert dec(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 32, 8, 64, 64, 65, scale, None, 0, STREAM) == 1
    assert dec(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 32, 8, 64, 64, 64, ctypes.c_float(float("inf")),
               None, 0, STREAM) == 1
    # prefill: nulls, empty, head_dim, a non-positive scale, rows beyond the cache
    pre = lib.mote_cuda_gqa_attention_prefill_f16
    assert pre(None, FAKE, FAKE, FAKE, 8, 0, 32, 8, 64, 0, 64, scale, STREAM) == 1
    assert pre(FAKE, FAKE, FAKE, FAKE, 0, 0, 32, 8, 64, 0, 64, scale, STREAM) == 0
    assert pre(FAKE, FAKE, FAKE, FAKE, 8, 0, 32, 8, 128, 0, 64, scale, STREAM) == 1
    assert pre(FAKE, FAKE, FAKE, FAKE, 8, 0, 32, 8, 64, 0, 64, ctypes.c_float(0.0), STREAM) == 1
    assert pre(FAKE, FAKE, FAKE, FAKE, 8, 0, 32, 8, 64, 0, 64, ctypes.c_float(-0.1), STREAM) == 1
    assert pre(FAKE, FAKE, FAKE, FAKE, 8, 60, 32, 8, 64, 0, 64, scale, STREAM) == 1


def test_decode_attention_chunk_plan(lib):
    """The decode split's chunk count (host logic): one chunk when the
    sequences x KV heads already fill the SMs, else chunks of whole tiles
    (2048 / head_dim positions) dealt eight to a CTA, where more than 8
    chunks (a cluster's worth, merged in the split kernel) cost four tiles
    more for the merge kernel; the workspace holds one f32 partial output plus max
    and sum per (sequence, query head, chunk)."""
    def ws(batch, qh, kvh, hd, max_len):
        n = ctypes.c_uint64(123)
        assert lib.mote_cuda_gqa_attention_decode_workspace_bytes(batch, qh, kvh, hd, max_len,
                                                                  ctypes.byref(n)) == 0
        return n.value
    assert ws(16, 32, 8, 64, 4096) == 0                  # 128 CTAs, one chunk each
    assert ws(1, 32, 8, 64, 4096) == 32 * 8 * 66 * 4     # 8 chunks of 16 tiles (a cluster)
    assert ws(1, 32, 8, 64, 1000) == 32 * 4 * 66 * 4     # 4 chunks of 8 tiles (a cluster)
    assert ws(1, 32, 8, 64, 32768) == 32 * 16 * 66 * 4   # 16 chunks of 64 tiles, merged
    assert ws(1, 64, 2, 128, 2000) == 64 * 8 * 130 * 4   # two head groups, 125 tiles of 16
    assert ws(4, 32, 8, 64, 0) == 0
    assert ws(1, 32, 8, 96, 64) == 0                     # rejected by the launch itself


def test_decoder_stack_argument_rules(lib):
    n = ctypes.c_uint64(0)
    assert lib.mote_cuda_q4_0_decoder_stack_workspace_bytes(2048, ctypes.byref(n)) == 0
    assert n.value == 256 + 16 * 2048
    eps = ctypes.c_float(1e-5)
    stack = lib.mote_cuda_q4_0_decoder_stack_f16
    ws_ok = 0x10000  # 256-byte aligned
    assert stack(None, 1, FAKE, 2048, 8192, 32, 8, 64, eps, ws_ok, n.value, STREAM) == 1
    assert stack(FAKE, 0, FAKE, 2048, 8192, 32, 8, 64, eps, ws_ok, n.value, STREAM) == 0
    assert stack(FAKE, 1, FAKE, 2000, 8192, 32, 8, 64, eps, ws_ok, n.value, STREAM) == 1
    assert stack(FAKE, 1, FAKE, 2048, 8192, 30, 8, 64, eps, ws_ok, n.value, STREAM) == 1
    assert stack(FAKE, 1, FAKE, 2048, 8192, 32, 8, 64, eps, ws_ok, n.value - 1, STREAM) == 1
    assert stack(FAKE, 1, FAKE, 2048, 8192, 32, 8, 64, ctypes.c_float(-1.0), ws_ok, n.value,
                 STREAM) == 1


def test_stream_wait_event_rejects_null_handles(lib):
    assert lib.mote_cuda_stream_wait_event(None, FAKE) == 1
    assert lib.mote_cuda_stream_wait_event(STREAM, None) == 1


def test_status_strings(lib):
    assert b"invalid" in lib.mote_cuda_status_string(-1).lower()
    assert lib.mote_cuda_status_string(1)


def test_comm_argument_rules(lib):
    f = lib.mote_cuda_all_gather_p2p_f16
    assert f(FAKE, FAKE, FAKE, FAKE, 12, 0, 1, STREAM) == 1  # count not a multiple of 8
    assert f(FAKE, FAKE, FAKE, FAKE, 16, 1, 1, STREAM) == 1  # rank >= nranks
    assert f(FAKE + 8, FAKE, FAKE, FAKE, 16, 0, 1, STREAM) == 1  # send not 16-byte aligned
    assert f(FAKE, None, FAKE, FAKE, 16, 0, 1, STREAM) == 1
    assert f(FAKE, FAKE, FAKE, FAKE, 16, 0, 1, None) == 1
    assert lib.mote_cuda_comm_all_gather_f16(None, FAKE, FAKE, 8, STREAM) == 1
    assert lib.mote_cuda_comm_destroy(None) == 0
    comm = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    assert lib.mote_cuda_comm_init(ctypes.byref(comm), 2, uid, 2) == 1
    assert lib.mote_cuda_comm_init(ctypes.byref(comm), 0, uid, 0) == 1
    assert lib.mote_cuda_ipc_get_handle(None, uid) == 1
    assert lib.mote_cuda_ipc_close_handle(None) == 1


def test_residual_argument_rules(lib):
    fn = lib.mote_cuda_quantized_linear_q4_0_f16_residual
    assert fn(FAKE, FAKE, None, FAKE, 1, 8, 32, STREAM) == 1
    assert fn(FAKE, FAKE, FAKE, FAKE, 1, 8, 33, STREAM) == 1
    assert fn(FAKE, FAKE, FAKE, FAKE, 0, 8, 32, STREAM) == 0


def test_fused_allgather_argument_rules(lib):
    fn = lib.mote_cuda_quantized_linear_q4_0_f16_allgather
    ok = (FAKE, FAKE, FAKE, FAKE, FAKE)
    assert fn(*ok, 1, 16, 256, 32, 2, 2, STREAM) == 1      # rank >= nranks
    assert fn(*ok, 1, 12, 256, 32, 0, 2, STREAM) == 1      # shard not a multiple of 16
    assert fn(*ok, 1, 16, 96, 32, 0, 2, STREAM) == 1       # K not a multiple of 256
    assert fn(*ok, 1, 16, 33, 32, 0, 2, STREAM) == 1       # K not a multiple of 32
    assert fn(FAKE, FAKE, None, FAKE, FAKE, 1, 16, 256, 32, 0, 2, STREAM) == 1
    assert fn(*ok, 0, 16, 256, 32, 0, 2, STREAM) == 0      # no rows: no launch


def test_fused_norm_argument_rules(lib):
    eps = ctypes.c_float(1e-5)
    lin = lib.mote_cuda_q4_0_rms_norm_linear_f16
    assert lin(FAKE, None, FAKE, FAKE, 1, 16, 256, eps, STREAM) == 1          # null gamma
    assert lin(FAKE, FAKE, FAKE, FAKE, 1, 16, 256, ctypes.c_float(float("nan")), STREAM) == 1
    assert lin(FAKE, FAKE, FAKE, FAKE, 1, 16, 256, ctypes.c_float(-1.0), STREAM) == 1
    assert lin(FAKE, FAKE + 2, FAKE, FAKE, 1, 16, 256, eps, STREAM) == 1      # gamma alignment
    assert lin(FAKE, FAKE, FAKE, FAKE, 0, 16, 256, eps, STREAM) == 0          # empty
    assert lin(FAKE, FAKE, FAKE, FAKE, 1, 16, 33, eps, STREAM) == 1           # K % 32
    gu = lib.mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16
    assert gu(FAKE, FAKE, FAKE, None, FAKE, 1, 16, 256, eps, STREAM) == 1    # null up
    qkv = lib.mote_cuda_q4_0_rms_norm_qkv_rope_f16
    assert qkv(FAKE, FAKE, FAKE, None, FAKE, FAKE, 1, 2, 1, 64, 256, eps, STREAM) == 1
    assert qkv(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 2, 1, 24, 256, eps, STREAM) == 1  # hd % 16
    assert qkv(FAKE, FAKE, FAKE, FAKE + 2, FAKE, FAKE, 1, 2, 1, 64, 256, eps, STREAM) == 1
    assert qkv(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 2, 1, 64, 256, eps, STREAM) == 0


def test_q8_0_argument_rules(lib):
    for fn in (lib.mote_cuda_quantized_linear_q8_0_f16, lib.mote_cuda_quantized_linear_q8_0_f16_f32out):
        assert fn(None, FAKE, FAKE, 1, 8, 32, STREAM) == 1       # null input
        assert fn(FAKE, FAKE, FAKE, 1, 8, 33, STREAM) == 1       # K % 32
        assert fn(FAKE, FAKE, FAKE, 1, 8, 32, None) == 1         # null stream
        assert fn(FAKE, FAKE, FAKE, 0, 8, 32, STREAM) == 0       # empty: no launch
        assert fn(FAKE, FAKE, FAKE, 1 << 20, 1 << 13, 32, STREAM) == 9  # rows*N > u32


def test_kquant_argument_rules(lib):
    for fn in (lib.mote_cuda_quantized_linear_q4_k_f16,
               lib.mote_cuda_quantized_linear_q4_k_f16_f32out,
               lib.mote_cuda_quantized_linear_q6_k_f16):
        assert fn(None, FAKE, FAKE, 1, 8, 256, STREAM) == 1      # null input
        assert fn(FAKE, FAKE, FAKE, 1, 8, 288, STREAM) == 1      # K % 256 (a Q4_0-legal K)
        assert fn(FAKE, FAKE, FAKE, 0, 8, 288, STREAM) == 1      # K % 256 checked before empty
        assert fn(FAKE, FAKE, FAKE, 1, 8, 256, None) == 1        # null stream
        assert fn(FAKE, FAKE, FAKE, 0, 8, 256, STREAM) == 0      # empty: no launch
        assert fn(FAKE, FAKE, FAKE, 1 << 20, 1 << 13, 256, STREAM) == 9  # rows*N > u32
    dq = lib.mote_cuda_kquant_dequantize_f32
    assert dq(2, None, FAKE, 1, 256, STREAM) == 1
    assert dq(1, FAKE, FAKE, 1, 256, STREAM) == 1                # Q4_0 is not a K-quant
    assert dq(3, FAKE, FAKE, 1, 320, STREAM) == 1                # k % 256
    assert dq(3, FAKE, FAKE, 1, 256, None) == 1
    assert dq(2, FAKE, FAKE, 0, 256, STREAM) == 0


def test_blaslt_argument_rules(lib):
    # null context / output: -1 before any library call (hipblaslt_shim.cpp:326-408)
    assert lib.mote_cuda_blaslt_create(None) == -1
    assert lib.mote_cuda_blaslt_matmul_f16_f32(None, 1, 1, 1, FAKE, FAKE, FAKE, FAKE, 64,
                                               STREAM) == -1
    assert lib.mote_cuda_blaslt_last_error(None) is None
    lib.mote_cuda_blaslt_destroy(None)


CRATE = Path(__file__).resolve().parents[1] / "mote-backend-cuda"


def test_rust_crate_binds_every_declared_symbol():
    """The committed Cargo crate (not compiled here: no cargo) declares every
    entry point of the header in src/ffi.rs, with the same number of
    parameters, and registers the same kernel table as mote_b200.kernel."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    c_arity = {}
    for name, args in re.findall(r"\b(mote_cuda_\w+)\s*\(([^)]*)\)\s*;", text):
        args = args.strip()
        c_arity[name] = 0 if args in ("", "void") else args.count(",") + 1
    ffi = (CRATE / "src" / "ffi.rs").read_text()
    rs_arity = {name: (0 if not args.strip() else args.count(",") + 1)
                for name, args in re.findall(r"pub fn (mote_cuda_\w+)\(([^)]*)\)", ffi)}
    assert rs_arity == c_arity
    kernel_rs = (CRATE / "src" / "kernel.rs").read_text()
    rows = re.findall(r'\("(\w+)", DType::(\w+), "(mote_cuda_\w+)", (\d+), call_\w+\)', kernel_rs)
    from mote_b200 import kernel

    table = {(op, dt.lower()): sym for op, dt, sym, _ in rows}
    assert table == {(op, dt.name.lower()): sym for (op, dt), sym in kernel.CUDA_KERNELS.items()}
    for _, _, sym, words in rows:
        assert int(words) == c_arity[sym], sym
    build = (CRATE / "build.rs").read_text()
    assert "compute_{arch},code=sm_{arch}" in build and '"100a"' in build
