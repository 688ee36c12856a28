"""ctypes binding of ``libmote_cuda.so``.

Loading fails loudly: there is no CPU fallback anywhere in this package.  If
the library is missing the import of any op raises
:class:`NativeLibraryMissing` with the build command to run.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from . import build as _build

LIB_PATH: Path = _build.LIB_PATH

P = ctypes.c_void_p
U64 = ctypes.c_uint64
U32 = ctypes.c_uint32
SZ = ctypes.c_size_t
I = ctypes.c_int
F = ctypes.c_float
D = ctypes.c_double

# name -> (restype, argtypes); must match include/mote_cuda.h exactly.
SIGNATURES: dict[str, tuple] = {
    # runtime shim
    "mote_cuda_get_device_count": (I, [ctypes.POINTER(I)]),
    "mote_cuda_set_device": (I, [I]),
    "mote_cuda_malloc": (I, [ctypes.POINTER(P), SZ]),
    "mote_cuda_free": (I, [P]),
    "mote_cuda_memcpy_host_to_device": (I, [P, P, SZ]),
    "mote_cuda_memcpy_device_to_host": (I, [P, P, SZ]),
    "mote_cuda_stream_create": (I, [ctypes.POINTER(P)]),
    "mote_cuda_stream_destroy": (I, [P]),
    "mote_cuda_stream_synchronize": (I, [P]),
    "mote_cuda_mem_get_info": (I, [ctypes.POINTER(SZ), ctypes.POINTER(SZ)]),
    "mote_cuda_memcpy_host_to_device_async": (I, [P, P, SZ, P]),
    "mote_cuda_memcpy_device_to_host_async": (I, [P, P, SZ, P]),
    "mote_cuda_memset_async": (I, [P, I, SZ, P]),
    "mote_cuda_host_alloc": (I, [ctypes.POINTER(P), SZ]),
    "mote_cuda_host_free": (I, [P]),
    "mote_cuda_event_create": (I, [ctypes.POINTER(P)]),
    "mote_cuda_event_destroy": (I, [P]),
    "mote_cuda_event_record": (I, [P, P]),
    "mote_cuda_event_elapsed_ms": (I, [ctypes.POINTER(F), P, P]),
    "mote_cuda_stream_wait_event": (I, [P, P]),
    "mote_cuda_device_status": (I, [ctypes.POINTER(ctypes.c_uint), I]),
    "mote_cuda_status_string": (ctypes.c_char_p, [I]),
    "mote_cuda_abi_version": (I, []),
    # Q4_0 linear
    "mote_cuda_quantized_linear_q4_0_f16": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q4_0_f16_f32out": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q4_0_f32": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q8_0_f16": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q8_0_f16_f32out": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q4_k_f16": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q4_k_f16_f32out": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q6_k_f16": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_kquant_dequantize_f32": (I, [I, P, P, U64, U64, P]),
    "mote_cuda_blaslt_create": (I, [ctypes.POINTER(P)]),
    "mote_cuda_blaslt_destroy": (None, [P]),
    "mote_cuda_blaslt_last_error": (ctypes.c_char_p, [P]),
    "mote_cuda_blaslt_matmul_f16_f32": (I, [P, U64, U64, U64, P, P, P, P, SZ, P]),
    "mote_cuda_quantized_linear_q4_0_f16_ws": (I, [P, P, P, U64, U64, U64, P, U64, P]),
    "mote_cuda_q4_0_linear_workspace_bytes": (I, [U64, U64, U64, ctypes.POINTER(U64)]),
    "mote_cuda_quantized_linear_q4_0_f16_noalloc": (I, [P, P, P, U64, U64, U64, P]),
    "mote_cuda_q4_0_gate_up_swiglu_f16": (I, [P, P, P, P, U64, U64, U64, P]),
    "mote_cuda_quantized_linear_q4_0_f16_residual": (I, [P, P, P, P, U64, U64, U64, P]),
    "mote_cuda_q4_0_rms_norm_linear_f16": (I, [P, P, P, P, U64, U64, U64, F, P]),
    "mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16": (I, [P, P, P, P, P, U64, U64, U64, F, P]),
    "mote_cuda_q4_0_rms_norm_qkv_rope_f16": (I, [P, P, P, P, P, P, U64, U64, U64, U64, U64, F,
                                                 P]),
    "mote_cuda_q4_0_decode_f32": (I, [P, P, U64, U64, P]),
    "mote_cuda_q4_0_encode_f32": (I, [P, P, U64, U64, P]),
    # layer kernels
    "mote_cuda_rms_norm_f16": (I, [P, P, P, U64, U64, F, P]),
    "mote_cuda_fused_add_rms_norm_f16": (I, [P, P, P, P, U64, U64, F, P]),
    "mote_cuda_rope_f16": (I, [P, P, P, P, U64, U64, U64, U64, U32, P]),
    "mote_cuda_rms_norm_rope_f16": (I, [P, P, P, P, P, P, P, P, P, U64, U64, U64, U64, U64,
                                        U32, F, P]),
    "mote_cuda_swiglu_f16": (I, [P, P, P, U64, P]),
    "mote_cuda_embedding_gather_f16": (I, [P, P, P, U64, U64, U64, P, P]),
    "mote_cuda_rope_cos_sin_f32": (I, [P, P, P, U64, U64, D, P]),
    # multi-GPU exchange
    "mote_cuda_kv_cache_append_f16": (I, [P, P, P, P, P, U64, U64, U64, U64, P, P]),
    "mote_cuda_gqa_attention_decode_workspace_bytes": (I, [U64, U64, U64, U64, U64,
                                                           ctypes.POINTER(U64)]),
    "mote_cuda_gqa_attention_decode_f16": (I, [P, P, P, P, P, U64, U64, U64, U64, U64, U64,
                                               ctypes.c_float, P, U64, P]),
    "mote_cuda_gqa_attention_prefill_f16": (I, [P, P, P, P, U64, U64, U64, U64, U64, U64, U64,
                                                ctypes.c_float, P]),
    "mote_cuda_q4_0_decoder_stack_workspace_bytes": (I, [U64, ctypes.POINTER(U64)]),
    "mote_cuda_q4_0_decoder_stack_f16": (I, [P, U32, P, U64, U64, U64, U64, U64, ctypes.c_float,
                                             P, U64, P]),
    "mote_cuda_comm_unique_id": (I, [P]),
    "mote_cuda_comm_init": (I, [ctypes.POINTER(P), I, P, I]),
    "mote_cuda_comm_init_timeout": (I, [ctypes.POINTER(P), I, P, I, U64]),
    "mote_cuda_comm_abort": (I, [P]),
    "mote_cuda_comm_all_gather_f16": (I, [P, P, P, U64, P]),
    "mote_cuda_comm_destroy": (I, [P]),
    "mote_cuda_ipc_get_handle": (I, [P, P]),
    "mote_cuda_ipc_open_handle": (I, [P, ctypes.POINTER(P)]),
    "mote_cuda_ipc_close_handle": (I, [P]),
    "mote_cuda_all_gather_p2p_f16": (I, [P, P, P, P, U64, U32, U32, P]),
    "mote_cuda_all_gather_p2p_f16_timeout": (I, [P, P, P, P, U64, U32, U32, U64, P]),
    "mote_cuda_peer_flags_reset": (I, [P, U32, P]),
    "mote_cuda_quantized_linear_q4_0_f16_allgather": (I, [P, P, P, P, P, U64, U64, U64, U64, U32,
                                                          U32, P]),
}


class NativeLibraryMissing(RuntimeError):
    pass


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library with every signature declared."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is not built; run `python -m mote_b200.build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(status: int) -> str:
    s = lib().mote_cuda_status_string(int(status))
    return s.decode() if s else f"status {status}"
