"""ctypes binding of libhexcuda's C ABI (include/hexcuda.h).

The shared library is built in-tree (hexkernels_b200/libhexcuda.so) by
``make -C hexkernels_b200/csrc``.  Loading fails loudly when it is missing:
there is no CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libhexcuda.so"

P = C.c_void_p
I = C.c_int
I32 = C.c_int32
I64 = C.c_int64
U8 = C.c_uint8
I8 = C.c_int8
F = C.c_float
SZ = C.c_size_t

# name -> (restype, argtypes); mirrors include/hexcuda.h
SIGNATURES: dict[str, tuple] = {
    "hexcuda_init": (I, [I]),
    "hexcuda_init_devices": (I, [P, I]),
    "hexcuda_shutdown": (None, []),
    "hexcuda_device_count": (I, []),
    "hexcuda_device_ordinal": (I, [I]),
    "hexcuda_alloc": (P, [I, SZ]),
    "hexcuda_free": (I, [I, P]),
    "hexcuda_host_alloc": (P, [SZ]),
    "hexcuda_host_free": (I, [P]),
    "hexcuda_h2d": (I, [I, P, P, SZ]),
    "hexcuda_d2h": (I, [I, P, P, SZ]),
    "hexcuda_memset": (I, [I, P, I, SZ]),
    "hexcuda_sync": (I, [I]),
    "hexcuda_stream": (P, [I]),
    "hexcuda_set_stream": (I, [I, P]),
    "hexcuda_reset_stream": (I, [I]),
    "hexcuda_last_error": (I, []),
    "hexcuda_last_error_string": (C.c_char_p, []),
    "hexcuda_set_timing": (I, [I]),
    "hexcuda_last_kernel_ms": (F, []),
    "hexcuda_launch_count": (C.c_uint64, []),
    "hexcuda_mechanisms": (C.c_uint, [I]),
    # multi-GPU: shards and replicated outputs
    "hexcuda_shard_rows": (I, [I64, I, I, P, P]),
    "hexcuda_set_replicate": (I, [I]),
    "hexcuda_get_replicate": (I, []),
    "hexcuda_replica": (I, [I, P, P]),
    "hexcuda_last_collective_ms": (F, []),
    "hexcuda_allgather_rows": (I, [P, P, I64, SZ]),
    "hexcuda_comm_unique_id": (I, [P, SZ]),
    "hexcuda_comm_init_rank": (I, [I, I, P, SZ]),
    "hexcuda_comm_destroy": (I, []),
    "hexcuda_comm_allgather_rows": (I, [P, P, I64, SZ]),
    # device-pointer launchers
    "hexcuda_softmax_f32": (I, [I, P, P, I, I]),
    "hexcuda_softmax_f16": (I, [I, P, P, I, I]),
    "hexcuda_layernorm_f32": (I, [I, P, P, P, P, I, I, F]),
    "hexcuda_layernorm_f16": (I, [I, P, P, P, P, I, I, F]),
    "hexcuda_rmsnorm_f32": (I, [I, P, P, P, I, I, F]),
    "hexcuda_rmsnorm_f16": (I, [I, P, P, P, I, I, F]),
    "hexcuda_rmsnorm_gain_f16": (I, [I, P, P, P, I, I, F]),
    "hexcuda_rowreduce_f32": (I, [I, P, P, I, I, I]),
    "hexcuda_requant_per_channel": (I, [I, P, P, I, I, P, P, I8]),
    "hexcuda_requantize_i32_u8": (I, [I, P, P, I64, I32, I, U8]),
    "hexcuda_gemm_i8_requant": (I, [I, P, P, P, I, I, I, I32, I, I8]),
    "hexcuda_gemm_i8_bias_requant": (I, [I, P, P, P, P, I, I, I, I32, I, I8]),
    "hexcuda_gemm_i8_zp": (I, [I, P, P, P, I, I, I, I32, I32, I]),
    "hexcuda_gemm_u8s8_pc": (I, [I, P, P, P, P, I, I, I, I32, P, P, U8]),
    "hexcuda_gemm_hmx": (I, [I, P, P, I, P, P, I, I, I, I, I32]),
    "hexcuda_gemm_i8_rq_ex": (I, [I, P, P, I, P, P, P, I, I, I, I32, I, I8, I]),
    "hexcuda_gemm_i8_acc": (I, [I, P, I, P, I, P, P, I, P, P, I, I, I, I, I]),
    "hexcuda_ffn_relu_i8": (I, [I, P, P, P, P, P, P, I, I, I, I, I32, I, I8]),
    "hexcuda_gemm_hmx_s8u8": (I, [I, P, P, P, I, I, I, I]),
    "hexcuda_gemm_f16_ex": (I, [I, P, P, I, P, P, P, I, I, F, I, I, I]),
    "hexcuda_attn_lut_i8": (I, [I, I, P, P, P, P, P, P, I, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_attn_lut_i8_window": (I, [I, P, P, P, P, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_kv_cache_update_i8": (I, [I, P, P, P, P, I, I, I, I]),
    "hexcuda_rope_pair_f16": (I, [I, P, P, P, P, I64]),
    "hexcuda_gemm_i16": (I, [I, P, P, P, I, I, I]),
    "hexcuda_conv2d_hmx": (I, [I, P, P, P, P, I, I, I, I, I, I, I, I, I]),
    "hexcuda_mix_mlp_i8": (I, [I, P, P, P, P, P, P, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_token_mix_i8": (I, [I, P, P, P, P, P, P, I, I, I, I32, I, I32, I]),
    "hexcuda_rnn_cell_i8": (I, [I, P, P, P, P, P, P, I, I, I32, I, I8, P]),
    "hexcuda_affine_ew": (I, [I, P, I, P, I, I64, I32, I32, I64, I, I, I, I, I32, I32]),
    "hexcuda_ffn_hmx_i8": (I, [I, P, P, P, P, P, P, I, I, I, I, I]),
    "hexcuda_ffn_swiglu_hmx_i8": (I, [I, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I]),
    "hexcuda_encoder_block_i8": (I, [I, P, P, P, P, P, P, P, I, I, I]),
    "hexcuda_decoder_block_i8": (I, [I, P, P, P, P, P, P, P, P, I, I, I]),
    "hexcuda_attn_qkt_av_hmx": (I, [I, P, P, P, P, I, I, I]),
    "hexcuda_requant_ew": (I, [I, P, I, P, I, P, I64, I, I64, I32, I, I, I, I, I, I, I, P]),
    "hexcuda_epilogue_bias_i32": (I, [I, P, P, P, I, I]),
    "hexcuda_relu_i8": (I, [I, P, P, I64]),
    "hexcuda_reduce_int": (I, [I, P, P, I, I64, I, P]),
    "hexcuda_minmax_ew": (I, [I, P, P, I32, I, I, P, I64]),
    "hexcuda_group_sum_i8": (I, [I, P, P, I64, I]),
    "hexcuda_group_dot_i8": (I, [I, P, P, P, I64, I]),
    "hexcuda_gate_mul_requant_i8": (I, [I, P, P, P, P, I64, I32, I]),
    "hexcuda_ffn_lut_i8": (I, [I, P, P, P, P, P, P, P, I, I, I, I, I32, I, I8]),
    "hexcuda_scan_max_i8": (I, [I, P, P, I64]),
    "hexcuda_head_group_reduce_i8": (I, [I, P, P, I, I, I64, I32, I]),
    "hexcuda_layernorm_lut_i8": (I, [I, P, P, P, P, I, I, P, P, P, I]),
    "hexcuda_layernorm_lut_i16": (I, [I, P, P, I, I, P, P, P, I]),
    "hexcuda_lut_softmax_u8": (I, [I, P, P, I, I, P, P]),
    "hexcuda_lut_softmax_i16": (I, [I, P, P, I, I, P]),
    "hexcuda_requant_i16": (I, [I, P, P, I64, I32, I]),
    "hexcuda_norm_requant_i8": (I, [I, P, P, I64, I, P, P, I32, I, I]),
    "hexcuda_gemm_softmax_u8": (I, [I, P, P, I, P, P, I, I, I, I, I32, I]),
    "hexcuda_gelu_ffn_residual_i8": (I, [I, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I]),
    "hexcuda_gemm_hmx_ex": (I, [I, P, P, I, P, P, I, P, P, I, I, I, I, I, I, I32]),
    "hexcuda_gemm_u8s8_pc_noalloc": (I, [I, P, P, P, P, I, I, I, I32, P, P, U8]),
    "hexcuda_gemm_f16_nt": (I, [I, P, P, P, I, I, I]),
    "hexcuda_gemm_f16_nn": (I, [I, P, P, P, I, I, I]),
    "hexcuda_attn_f16": (I, [I, P, P, P, P, I, I, I, I, F, I]),
    "hexcuda_online_softmax_step_f16": (I, [I, P, P, P, P, P, I, I]),
    "hexcuda_selftest_watchdog": (I, [I, C.c_uint32]),
    # host-pointer entries
    "hexcuda_host_softmax_f32": (I, [P, P, I, I]),
    "hexcuda_host_softmax_f16": (I, [P, P, I, I]),
    "hexcuda_host_layernorm_f32": (I, [P, P, P, P, I, I, F]),
    "hexcuda_host_layernorm_f16": (I, [P, P, P, P, I, I, F]),
    "hexcuda_host_rmsnorm_f16": (I, [P, P, P, I, I, F]),
    "hexcuda_host_rmsnorm_gain_f16": (I, [P, P, P, I, I, F]),
    "hexcuda_host_rowreduce_f32": (I, [P, P, I, I, I]),
    "hexcuda_host_requant_per_channel": (I, [P, P, I, I, P, P, I8]),
    "hexcuda_host_requantize_i32_u8": (I, [P, P, I64, I32, I, U8]),
    "hexcuda_host_gemm_i8_requant": (I, [P, P, P, I, I, I, I32, I, I8]),
    "hexcuda_host_gemm_i8_bias_requant": (I, [P, P, P, P, I, I, I, I32, I, I8]),
    "hexcuda_host_gemm_i8_zp": (I, [P, P, P, I, I, I, I32, I32, I]),
    "hexcuda_host_gemm_u8s8_pc": (I, [P, P, P, P, I, I, I, I32, P, P, U8]),
    "hexcuda_host_gemm_hmx": (I, [P, P, I, P, P, I, I, I, I, I32]),
    "hexcuda_host_gemm_i8_rq_ex": (I, [P, P, I, P, P, P, I, I, I, I32, I, I8, I]),
    "hexcuda_host_gemm_i8_acc": (I, [P, I, P, I, P, P, I, P, P, I, I, I, I, I]),
    "hexcuda_host_ffn_relu_i8": (I, [P, P, P, P, P, P, I, I, I, I, I32, I, I8]),
    "hexcuda_host_gemm_hmx_s8u8": (I, [P, P, P, I, I, I, I]),
    "hexcuda_host_gemm_f16_ex": (I, [P, P, I, P, P, P, I, I, F, I, I, I]),
    "hexcuda_host_attn_lut_i8": (I, [I, P, P, P, P, P, P, I, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_host_attn_lut_i8_window": (I, [P, P, P, P, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_host_kv_cache_update_i8": (I, [P, P, P, P, I, I, I, I]),
    "hexcuda_host_rope_pair_f16": (I, [P, P, P, P, I64]),
    "hexcuda_host_gemm_i16": (I, [P, P, P, I, I, I]),
    "hexcuda_host_conv2d_hmx": (I, [P, P, P, P, I, I, I, I, I, I, I, I, I]),
    "hexcuda_host_mix_mlp_i8": (I, [P, P, P, P, P, P, P, I, I, I, I, I32, I, I32, I]),
    "hexcuda_host_token_mix_i8": (I, [P, P, P, P, P, P, I, I, I, I32, I, I32, I]),
    "hexcuda_host_rnn_cell_i8": (I, [P, P, P, P, P, P, I, I, I32, I, I8, P]),
    "hexcuda_host_affine_ew": (I, [P, I, P, I, I64, I32, I32, I64, I, I, I, I, I32, I32]),
    "hexcuda_host_ffn_hmx_i8": (I, [P, P, P, P, P, P, I, I, I, I, I]),
    "hexcuda_host_ffn_swiglu_hmx_i8": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, I, I]),
    "hexcuda_host_encoder_block_i8": (I, [P, P, P, P, P, P, P, I, I, I]),
    "hexcuda_host_decoder_block_i8": (I, [P, P, P, P, P, P, P, P, I, I, I]),
    "hexcuda_host_attn_qkt_av_hmx": (I, [P, P, P, P, I, I, I]),
    "hexcuda_host_requant_ew": (I, [P, I, P, I, P, I64, I, I64, I32, I, I, I, I, I, I, I, P]),
    "hexcuda_host_epilogue_bias_i32": (I, [P, P, P, I, I]),
    "hexcuda_host_relu_i8": (I, [P, P, I64]),
    "hexcuda_host_reduce_int": (I, [P, P, I, I64, I, P]),
    "hexcuda_host_minmax_ew": (I, [P, P, I32, I, I, P, I64]),
    "hexcuda_host_group_sum_i8": (I, [P, P, I64, I]),
    "hexcuda_host_group_dot_i8": (I, [P, P, P, I64, I]),
    "hexcuda_host_gate_mul_requant_i8": (I, [P, P, P, P, I64, I32, I]),
    "hexcuda_host_ffn_lut_i8": (I, [P, P, P, P, P, P, P, I, I, I, I, I32, I, I8]),
    "hexcuda_host_scan_max_i8": (I, [P, P, I64]),
    "hexcuda_host_head_group_reduce_i8": (I, [P, P, I, I, I64, I32, I]),
    "hexcuda_host_layernorm_lut_i8": (I, [P, I, P, P, P, I, I, P, P, P, I]),
    "hexcuda_host_layernorm_lut_i16": (I, [P, P, I, I, P, P, P, I]),
    "hexcuda_host_lut_softmax_u8": (I, [P, P, I, I, P, P]),
    "hexcuda_host_lut_softmax_i16": (I, [P, P, I, I, P]),
    "hexcuda_host_requant_i16": (I, [P, P, I64, I32, I]),
    "hexcuda_host_norm_requant_i8": (I, [P, P, I64, I, P, P, I32, I, I]),
    "hexcuda_host_gemm_softmax_u8": (I, [P, P, I, P, P, I, I, I, I, I32, I]),
    "hexcuda_host_gelu_ffn_residual_i8": (I, [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I]),
    "hexcuda_host_gemm_hmx_ex": (I, [P, P, I, P, P, I, P, P, I, I, I, I, I, I, I32]),
    "hexcuda_host_gemm_f16_nt": (I, [P, P, P, I, I, I]),
    "hexcuda_host_gemm_f16_nn": (I, [P, P, P, I, I, I]),
    "hexcuda_host_attn_f16": (I, [P, P, P, P, I, I, I, I, F, I]),
    "hexcuda_host_online_softmax_step_f16": (I, [P, P, P, P, P, I, I]),
}

ERRORS = {0: "OK", 1: "ERR_ARG", 2: "ERR_CUDA", 3: "ERR_NODEV", 4: "ERR_TIMEOUT", 5: "ERR_OOM"}

_lib = None


class HexcudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"hexcuda {ERRORS.get(code, code)}: {msg}")
        self.code = code


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load libhexcuda.so and declare every exported signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `make -C {PKG_DIR / 'csrc'}` "
            "(the operators have no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != 0:
        lib = load()
        raise HexcudaError(rc, lib.hexcuda_last_error_string().decode(errors="replace"))
