"""ctypes binding of the C ABI in ``include/qwen35_b200.h`` (``ppu_b200/_lib/libqwen35_b200.so``).

There is no CPU fallback: if the library is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libqwen35_b200.so"

Q35_OK, Q35_EINVAL, Q35_ECUDA, Q35_ETIMEOUT, Q35_ENOTSUP = 0, 1, 2, 3, 4
PRO_PLAIN, PRO_NORM, PRO_EMBED = 0, 1, 2
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2
EPI_BIAS, EPI_BIAS_GELU_TANH, EPI_BIAS_GELU = 3, 4, 5
Q35_GEMV_BULK, Q35_GEMV_REGISTERS = 0, 1

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32
F32 = C.c_float
SZ = C.c_size_t
INT = C.c_int


class GemvDesc(C.Structure):
    _fields_ = [
        ("weight", P), ("w_scale", P), ("input", P), ("norm_weight", P), ("token", P), ("embed", P),
        ("resid_out", P), ("out", P), ("n_out", I64), ("k", I64), ("vocab", I64),
        ("prologue", I32), ("epilogue", I32), ("int8", I32), ("eps", F32),
    ]


class LayerDesc(C.Structure):
    _fields_ = [
        ("kind", I32), ("in_ln", P), ("post_ln", P), ("mix_in", P), ("mix_in_scale", P), ("mix_out", P),
        ("mix_out_scale", P), ("gate_up", P), ("gate_up_scale", P), ("down", P), ("down_scale", P),
        ("conv_w", P), ("a_log", P), ("dt_bias", P), ("gnorm", P), ("conv_state", P), ("rec_state", P),
        ("q_norm", P), ("k_norm", P), ("k_cache", P), ("v_cache", P),
    ]


class DecoderDesc(C.Structure):
    _fields_ = [
        ("n_layers", I32), ("hidden", I32), ("intermediate", I32), ("vocab", I32),
        ("q_heads", I32), ("kv_heads", I32), ("head_dim", I32), ("rotary_dim", I32),
        ("lin_heads", I32), ("lin_dk", I32), ("lin_dv", I32), ("conv_kernel", I32), ("delta_rows", I32),
        ("max_len", I32), ("max_prefill", I32), ("a8w8", I32), ("eps", F32),
        ("layers", C.POINTER(LayerDesc)), ("embed", P), ("final_norm", P), ("inv_freq", P),
        ("token", P), ("cache_len", P), ("rope_pos", P), ("token_log", P), ("log_pos", P),
        ("log_len", I32), ("use_pdl", I32), ("prefill_tc", I32), ("prefill_delta", I32),
        ("mrope_section", I32 * 3), ("batch", I32), ("workspace", P), ("workspace_bytes", SZ),
    ]


class VitBlockDesc(C.Structure):
    _fields_ = [
        ("norm1_w", P), ("norm1_b", P), ("qkv_w", P), ("qkv_b", P), ("proj_w", P), ("proj_b", P),
        ("norm2_w", P), ("norm2_b", P), ("fc1_w", P), ("fc1_b", P), ("fc2_w", P), ("fc2_b", P),
    ]


class VitDesc(C.Structure):
    _fields_ = [
        ("depth", I32), ("width", I32), ("heads", I32), ("intermediate", I32),
        ("in_channels", I32), ("patch", I32), ("temporal_patch", I32), ("merge", I32),
        ("out_width", I32), ("pos_side", I32), ("max_patches", I32), ("eps", F32),
        ("pixel_mean", F32), ("pixel_std", F32),
        ("blocks", C.POINTER(VitBlockDesc)), ("patch_w", P), ("patch_b", P), ("pos_table", P), ("rope_inv_freq", P),
        ("merger_norm_w", P), ("merger_norm_b", P), ("merger_fc1_w", P), ("merger_fc1_b", P),
        ("merger_fc2_w", P), ("merger_fc2_b", P), ("workspace", P), ("workspace_bytes", SZ),
    ]


_SIGS = {
    "q35_last_error": (C.c_char_p, []),
    "q35_abi_version": (INT, []),
    "q35_rms_norm": (INT, [P, P, P, I64, I64, F32, P]),
    "q35_residual_add_rms_norm": (INT, [P, P, P, P, P, I64, I64, F32, P]),
    "q35_gated_rms_norm": (INT, [P, P, P, P, I64, I64, F32, P]),
    "q35_silu_and_mul": (INT, [P, P, I64, I64, P]),
    "q35_sigmoid_mul": (INT, [P, P, P, I64, P]),
    "q35_attention_gate_mul": (INT, [P, P, P, I64, I64, I64, I64, P]),
    "q35_embedding": (INT, [P, P, P, I64, I64, I64, P]),
    "q35_swiglu_gemv": (INT, [P, P, P, I64, I64, P]),
    "q35_gemv": (INT, [C.POINTER(GemvDesc), P]),
    "q35_set_gemv_variant": (INT, [INT]),
    "q35_gemv_error": (INT, []),
    "q35_lm_head_workspace_size": (SZ, [I64]),
    "q35_lm_head_argmax": (INT, [P, P, P, P, I64, I64, I64, F32, P, SZ, P]),
    "q35_lm_shard_workspace_size": (SZ, []),
    "q35_lm_head_shard_keys": (INT, [P, I64, P, P, I64, I64, I64, I64, F32, P, P, SZ, P]),
    "q35_lm_keys_to_tokens": (INT, [P, I64, P, P]),
    "q35_quantize_rows": (INT, [P, P, P, I64, I64, P]),
    "q35_quantize_tokens": (INT, [P, P, P, I64, I64, P]),
    "q35_a8w8_linear_workspace_size": (SZ, [I64, I64]),
    "q35_a8w8_linear": (INT, [P, P, P, P, I64, I64, I64, P, SZ, P]),
    "q35_int8_gemm_i32": (INT, [P, P, P, I64, I64, I64, P]),
    "q35_gemm_bf16": (INT, [P, P, P, I64, I64, I64, I32, P]),
    "q35_gemm_tc": (INT, [P, P, P, I64, I64, I64, I32, P]),
    "q35_gemm_tc_a8w8": (INT, [P, P, P, P, P, I64, I64, I64, I32, P]),
    "q35_tc_error": (INT, []),
    "q35_set_gemm_tc_pairs": (INT, [C.c_int]),
    "q35_delta_chunk_error": (INT, []),
    "q35_qgkv_norm_rope": (INT, [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, F32, P]),
    "q35_gqa_decode_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "q35_gqa_decode_attention": (INT, [P, P, P, P, F32, P, I64, I64, I64, I64, I64, P, SZ, P]),
    "q35_gqa_decode_noalloc_max_bytes": (SZ, []),
    "q35_gqa_decode_attention_noalloc": (INT, [P, P, P, P, F32, P, I64, I64, I64, I64, I64, P]),
    "q35_attn_decode_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "q35_attn_decode": (INT, [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, F32, P, SZ, P]),
    "q35_prefill_attention": (INT, [P, P, P, P, I64, I64, I64, I64, I64, I64, I64, F32, P]),
    "q35_prefill_attention_tc": (INT, [P, P, P, P, I64, I64, I64, I64, I64, I64, F32, P, SZ, P]),
    "q35_prefill_attention_tc_workspace_size": (SZ, [I64, I64, I64]),
    "q35_prefill_attention_tc_error": (INT, []),
    "q35_causal_conv1d": (INT, [P, P, P, P, I64, I64, I64, I64, I64, P]),
    "q35_delta_recurrent": (INT, [P, P, P, P, P, P, I64, I64, I64, I64, I64, P]),
    "q35_delta_decode": (INT, [P, P, P, P, P, P, P, P, I64, I64, I64, I64, F32, P]),
    "q35_delta_chunked_workspace_size": (SZ, [I64, I64, I64]),
    "q35_delta_chunked": (INT, [P, P, P, P, P, P, I64, I64, I64, I64, I64, P, SZ, P]),
    "q35_delta_chunked_conv": (INT, [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, P, SZ, P]),
    "q35_decoder_workspace_size": (SZ, [C.POINTER(DecoderDesc)]),
    "q35_decoder_create": (INT, [C.POINTER(DecoderDesc), C.POINTER(P)]),
    "q35_decoder_destroy": (None, [P]),
    "q35_decoder_prefill": (INT, [P, P, I64, P]),
    "q35_decoder_prefill_mm": (INT, [P, P, I64, P, P, I64, P, I64, I64, P]),
    "q35_decoder_prefill_slot": (INT, [P, P, I64, I64, P]),
    "q35_decoder_prefill_batch": (INT, [P, P, I64, I64, P, P, I64, P, I64, I64, P]),
    "q35_gemv_batch": (INT, [C.POINTER(GemvDesc), I64, P]),
    "q35_decoder_decode_step": (INT, [P, P]),
    "q35_decoder_decode_layers": (INT, [P, P]),
    "q35_decoder_hidden": (P, [P]),
    "q35_decoder_finish_step": (INT, [P, P, I64, P]),
    "q35_decoder_kernels_per_step": (INT, [P]),
    "q35_decoder_decode_step_persistent": (INT, [P, P]),
    "q35_decoder_has_persistent": (INT, [P]),
    "q35_set_gemv_ctas_per_sm": (INT, [C.c_int]),
    "q35_decoder_set_trace": (INT, [P, P, I64]),
    "q35_decoder_trace_ops": (INT, [P]),
    "q35_decoder_set_probe": (INT, [P, P, SZ]),
    "q35_gemm_tc_bias": (INT, [P, P, P, P, I64, I64, I64, I32, P]),
    "q35_layer_norm": (INT, [P, P, P, P, I64, I64, F32, P]),
    "q35_residual_add_layer_norm": (INT, [P, P, P, P, P, P, I64, I64, F32, P]),
    "q35_position_embed_add": (INT, [P, P, P, P, P, I64, I64, I64, P]),
    "q35_vision_qkv_rope": (INT, [P, P, P, P, P, P, I64, I64, I64, P]),
    "q35_vision_attention": (INT, [P, P, P, P, I64, I64, I64, F32, P]),
    "q35_vision_rope_table": (INT, [P, P, P, I64, I64, I64, P]),
    "q35_vision_patchify": (INT, [P, P, I64, I64, I64, I64, I64, I64, F32, F32, P]),
    "q35_vit_workspace_size": (SZ, [C.POINTER(VitDesc)]),
    "q35_vit_create": (INT, [C.POINTER(VitDesc), C.POINTER(P)]),
    "q35_vit_destroy": (None, [P]),
    "q35_vit_encode": (INT, [P, P, I64, I64, P, P]),
    "q35_vit_encode_batch": (INT, [P, P, I64, I64, I64, P, P]),
    "q35_vit_encode_patches": (INT, [P, P, I64, I64, P, P]),
    "q35_vit_hidden": (P, [P]),
    "q35_decoder_probe_bytes": (SZ, [P]),
    "q35_decoder_persistent_error": (INT, []),
}

EXPORTED = tuple(_SIGS)

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m ppu_b200.build` "
                "(there is no CPU fallback for the fused operators)"
            )
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    return load().q35_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Map a C status to the reference's exception types (ValueError for bad arguments)."""
    if rc == Q35_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (Q35_EINVAL, Q35_ENOTSUP):
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_of(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
