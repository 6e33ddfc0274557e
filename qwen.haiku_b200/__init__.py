# SPDX-License-Identifier: MIT
"""qwen.haiku_b200 -- B200 (sm_100a) backend for qwen.haiku's quantized
matmul path, loaded from the in-tree C-ABI library libqh200.so.

The package directory name contains a dot, so it is loaded by path (see
``load()`` in tests/conftest.py, bench.py and __graft_entry__.py); inside it
everything is plain relative imports.

Python here is glue: ctypes bindings of include/qh_backend.h and
include/qh_synth.h, plus a thin mirror of the reference's matmul interface
(slm/tensor.c:827-1033, slm/model.c:220) over device buffers for tests and
benchmarks. All arithmetic runs in the CUDA kernels of libqh200.so; there is
no CPU fallback -- calls fail loudly when the library or a GPU is missing.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqh200.so")

# Status codes (include/qh_backend.h).
QH_OK = 0
STATUS_NAMES = {
    -1: "QH_ERR_INVALID", -2: "QH_ERR_UNSUPPORTED", -3: "QH_ERR_CUDA",
    -4: "QH_ERR_ALIGN", -5: "QH_ERR_WORKSPACE", -6: "QH_ERR_DEVICE",
}

# qh_slm_set_prefill_mode, qh_slm_set_decode_mode (include/qh_slm.h)
PREFILL_STEPWISE, PREFILL_CHUNKED = 0, 1
DECODE_PERSISTENT, DECODE_LAUNCHES = 0, 1

# GGUF tensor types (slm/gguf.c:52-59).
F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
TYPE_NAMES = {F32: "F32", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34}
BLOCK_WEIGHTS = {Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_0: 32}


class GemmJob(C.Structure):
    """qh_gemm_job (include/qh_backend.h)."""
    _fields_ = [("d_wt", C.c_void_p), ("out_f", C.c_int64), ("d_out", C.c_void_p), ("ld_out", C.c_int64)]


# qh_step_* (include/qh_kernels.h): persistent decode-step programs.
STEP_MATVEC, STEP_GDN, STEP_ATTN = 0, 1, 2
STEP_X_RESNORM, STEP_X_SWIGLU, STEP_X_QUANT = 1, 2, 3
STEP_MAX_PROJ = 8


class StepProj(C.Structure):
    """qh_step_proj (include/qh_kernels.h)."""
    _fields_ = [("type", C.c_int32), ("d_w", C.c_void_p), ("k", C.c_int64), ("out_f", C.c_int64),
                ("d_out", C.c_void_p)]


class StepPhase(C.Structure):
    """qh_step_phase (include/qh_kernels.h)."""
    _fields_ = [("kind", C.c_int32), ("xform", C.c_int32), ("xk", C.c_int64), ("eps", C.c_float),
                ("d_xa", C.c_void_p), ("d_xb", C.c_void_p), ("d_xw", C.c_void_p), ("d_xh_out", C.c_void_p),
                ("n_proj", C.c_int32), ("proj", StepProj * STEP_MAX_PROJ), ("d_act_out", C.c_void_p),
                ("d_qkv", C.c_void_p), ("d_ring", C.c_void_p), ("d_conv_w", C.c_void_p), ("d_b", C.c_void_p),
                ("d_a", C.c_void_p), ("d_dt_bias", C.c_void_p), ("d_ssm_a", C.c_void_p), ("d_state", C.c_void_p),
                ("d_z", C.c_void_p), ("d_norm_w", C.c_void_p), ("d_y", C.c_void_p),
                ("heads", C.c_int32), ("head_dim", C.c_int32), ("conv_kernel", C.c_int32),
                ("d_qraw", C.c_void_p), ("d_kin", C.c_void_p), ("d_vin", C.c_void_p), ("d_qnorm_w", C.c_void_p),
                ("d_knorm_w", C.c_void_p), ("d_rope", C.c_void_p), ("d_kcache", C.c_void_p),
                ("d_vcache", C.c_void_p), ("d_ctx", C.c_void_p), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("rope_dim", C.c_int32), ("max_pos", C.c_int32)]


class QHError(RuntimeError):
    """A libqh200 call returned a non-zero status."""

    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class MatvecJob(C.Structure):
    _fields_ = [("d_w", C.c_void_p), ("d_xq", C.c_void_p), ("d_out", C.c_void_p),
                ("k", C.c_int64), ("out_f", C.c_int64),
                ("xq_rows", C.c_int64), ("xq_row0", C.c_int64)]


_P, _I, _I64, _U64, _F, _SZ = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float, C.c_size_t


class Sampler(C.Structure):
    """qh_sampler (include/qh_sampler.h) = struct slm_sampler."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repetition_penalty", C.c_float), ("repetition_window", C.c_int32)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}

# name -> (restype, argtypes); every declaration of include/qh_backend.h and
# include/qh_synth.h.
SIGNATURES = {
    "qh_version": (C.c_char_p, []),
    "qh_last_error": (C.c_char_p, []),
    "qh_device_count": (_I, []),
    "qh_set_device": (_I, [_I]),
    "qh_malloc": (_I, [C.POINTER(C.c_void_p), _SZ]),
    "qh_free": (_I, [_P]),
    "qh_memcpy_h2d": (_I, [_P, _P, _SZ, _P]),
    "qh_memcpy_d2h": (_I, [_P, _P, _SZ, _P]),
    "qh_memset": (_I, [_P, _I, _SZ, _P]),
    "qh_stream_sync": (_I, [_P]),
    "qh_check_device_error": (_I, [C.POINTER(C.c_int)]),
    "qh_q8k_bytes": (_I64, [_I64, _I64]),
    "qh_q8_0_bytes": (_I64, [_I64, _I64]),
    "qh_q8k_d_offset": (_I64, [_I64, _I64]),
    "qh_q8k_bsums_offset": (_I64, [_I64, _I64]),
    "qh_q8_0_d_offset": (_I64, [_I64, _I64]),
    "qh_quantize_q8k": (_I, [_P, _I64, _I64, _P, _P]),
    "qh_quantize_q8_0": (_I, [_P, _I64, _I64, _P, _P]),
    "qh_matmul_workspace_bytes": (_I64, [_I, _I64, _I64]),
    "qh_matmul_q4k_f32": (_I, [_P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_matmul_q5k_f32": (_I, [_P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_matmul_q6k_f32": (_I, [_P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_matmul_q8_0_f32": (_I, [_P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_matmul_q4k_f32_noalloc": (_I, [_P, _I64, _I64, _P, _I64, _P, _P]),
    "qh_matmul_f32": (_I, [_P, _I64, _I64, _P, _I64, _P, _P]),
    "qh_matmul": (_I, [_I, _P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_matmul_preq": (_I, [_I, _P, _I64, _I64, _P, _I64, _P, _P]),
    "qh_matvec_plan_create": (_I, [_I, C.POINTER(MatvecJob), _I, _I64, C.POINTER(C.c_void_p)]),
    "qh_matvec_plan_run": (_I, [_P, _P]),
    "qh_matvec_plan_info": (_I, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "qh_matvec_plan_destroy": (_I, [_P]),
    "qh_matvec_plan_test_timeout": (_I, [_P, C.c_int32, C.c_uint32]),
    "qh_gemm_weight_bytes": (_I64, [_I, _I64, _I64]),
    "qh_gemm_pack_weights": (_I, [_I, _P, _I64, _I64, _P, _P]),
    "qh_gemm_expanded_bytes": (_I64, [_I, _I64, _I64]),
    "qh_matvec_plan_fuse_input": (_I, [_P, _I, _P, _P, _P, C.c_float, _P]),
    "qh_matvec_plan_fuse_output": (_I, [_P, _I, _I64, _P, _P, _P, C.c_float, _P, _P]),
    "qh_gemm_expand_weights": (_I, [_I, _P, _I64, _I64, _P, _P]),
    "qh_q8kt_bytes": (_I64, [_I64, _I64]),
    "qh_quantize_q8kt": (_I, [_P, _I64, _I64, _P, _P]),
    "qh_gemm_scratch_bytes": (_I64, [_P, _I, _I64, _I64]),
    "qh_gemm": (_I, [_I, _P, _I, _I64, _P, _I64, _P, _I64, C.c_int32, _P]),
    "qh_matmul_gemm_workspace_bytes": (_I64, [_I, _I64, _I64, _I64]),
    "qh_matmul_gemm": (_I, [_I, _P, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qh_synth_u64": (_U64, [_U64, _U64]),
    "qh_synth_normal": (_I, [_U64, _I64, _F, _F, _P]),
    "qh_synth_blocks": (_I, [_I, _I64, _U64, _P]),
    "qh_synth_quantize": (_I, [_I, _P, _I64, _I64, _P]),
}

class SlmConfig(C.Structure):
    """qh_slm_config (include/qh_slm.h)."""
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("ffn", C.c_int32), ("vocab", C.c_int32),
                ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("rope_dim", C.c_int32), ("rope_theta", C.c_float), ("rope_sections", C.c_int32 * 4),
                ("norm_eps", C.c_float), ("gdn_heads", C.c_int32), ("gdn_head_dim", C.c_int32),
                ("conv_kernel", C.c_int32), ("full_attn_interval", C.c_int32), ("max_pos", C.c_int32)]


SIGNATURES.update({
    "qh_slm_config_default": (None, [C.POINTER(SlmConfig), C.c_int32]),
    "qh_blob_synthetic": (_I, [C.POINTER(SlmConfig), _U64, C.POINTER(C.c_void_p)]),
    "qh_blob_synthetic_mix": (_I, [C.POINTER(SlmConfig), _U64, C.c_int32, C.POINTER(C.c_void_p)]),
    "qh_blob_count": (_I, [_P]),
    "qh_blob_tensor": (_I, [_P, _I, C.POINTER(C.c_char_p), C.POINTER(C.c_int32), C.POINTER(_I64),
                           C.POINTER(C.c_void_p), C.POINTER(_I64)]),
    "qh_blob_find": (_I, [_P, C.c_char_p]),
    "qh_blob_free": (None, [_P]),
    "qh_blob_create": (_I, [C.POINTER(C.c_void_p)]),
    "qh_blob_add": (_I, [_P, C.c_char_p, C.c_int32, C.POINTER(_I64), _P, _I64]),
    "qh_gguf_load": (_I, [C.c_char_p, C.c_int32, C.POINTER(SlmConfig), C.POINTER(C.c_void_p)]),
    "qh_gguf_write": (_I, [C.c_char_p, C.POINTER(SlmConfig), _P]),
    "qh_slm_create": (_I, [C.POINTER(SlmConfig), _P, C.c_int32, C.POINTER(C.c_void_p)]),
    "qh_slm_destroy": (None, [_P]),
    "qh_slm_reset": (_I, [_P]),
    "qh_slm_step": (_I, [_P, _P, C.c_int32, _P, _P]),
    "qh_slm_generate": (_I, [_P, _P, C.c_int32, C.c_int32, _P]),
    "qh_slm_memory": (_I, [_P, C.POINTER(_I64), C.POINTER(_I64)]),
    "qh_slm_begin": (_I, [_P, _P, C.c_int32]),
    "qh_slm_prefill": (_I, [_P, _P, C.c_int32]),
    "qh_slm_prefill_at": (_I, [_P, _P, C.c_int32, C.c_int32]),
    "qh_slm_position": (C.c_int32, [_P]),
    "qh_slm_sample_setup": (_I, [_P, C.POINTER(Sampler), _P, C.c_int32, C.c_int32, C.c_int32, _P, C.c_int32]),
    "qh_slm_sample_steps": (_I, [_P, C.c_int32, _P]),
    "qh_slm_set_prefill_chunk": (_I, [_P, C.c_int32]),
    "qh_slm_set_prefill_mode": (_I, [_P, C.c_int32]),
    "qh_slm_set_decode_mode": (_I, [_P, C.c_int32]),
    "qh_slm_decode_mode": (C.c_int32, [_P]),
    "qh_slm_step_stamps": (_I, [_P, _P]),
    "qh_slm_advance": (_I, [_P, C.c_int32]),
    "qh_slm_picks": (_I, [_P, C.c_int32, C.c_int32, _P]),
    "qh_slm_stream": (_P, [_P]),
    "qh_slm_device_next": (_P, [_P]),
})

_F32P = C.c_void_p
SIGNATURES.update({  # include/qh_kernels.h
    "qh_libm_eval": (_I, [_I, C.c_uint32, _I64, _P, _P]),
    "qh_step_create": (_I, [_P, C.c_int32, _P, _P]),
    "qh_step_run": (_I, [_P, C.c_int32, C.c_int32, _P]),
    "qh_step_destroy": (None, [_P]),
    "qh_step_set_stamps": (_I, [_P, _P]),
    "qh_step_phase_count": (C.c_int32, [_P]),
    "qh_step_test_timeout": (_I, [_P, C.c_int32, C.c_uint32]),
    "qh_embed_q6k": (_I, [_P, _I64, _P, C.c_int32, _P, _P]),
    "qh_embed_f32": (_I, [_P, _I64, _P, C.c_int32, _P, _P]),
    "qh_rmsnorm": (_I, [_P, _P, _I64, _I64, C.c_float, _P, _P]),
    "qh_add": (_I, [_P, _P, _I64, _P]),
    "qh_swiglu": (_I, [_P, _P, _P, _I64, _P]),
    "qh_gdn_pre": (_I, [_P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P,
                        _P, _P, _P, _P, _P, _P]),
    "qh_gdn_recurrence": (_I, [_P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, _P, _P]),
    "qh_gdn_gated_norm": (_I, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_float, _P, _P]),
    "qh_attn_pre": (_I, [_P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                         C.c_float, _P, C.c_int32, _P, _P, _P, _P, _P]),
    "qh_attn_decode": (_I, [_P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, C.c_int32,
                            _P, _P]),
    "qh_argmax": (_I, [_P, C.c_int32, _I64, _P, _P]),
    "qh_feed_next": (_I, [_P, _P, C.c_int32, C.c_int32, _P, _P, _P, _P]),
    "qh_rmsnorm_q8k": (_I, [_P, _P, _P, _P, _I64, C.c_int32, C.c_float, _P, C.c_int32, _P]),
    "qh_swiglu_q8k": (_I, [_P, _P, _I64, C.c_int32, _P, C.c_int32, _P]),
    "qh_gdn_fused": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                          C.c_float, _P, _P, C.c_int32, _P]),
    "qh_argmax_feed_scratch_bytes": (_I64, [C.c_int32, _I64]),
    "qh_gdn_fused_y": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                            C.c_float, _P, _P, _P]),
    "qh_attn_prefill_pre": (_I, [_P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                 C.c_int32, C.c_float, _P, C.c_int32, _P, _P, _P, _P, _P]),
    "qh_attn_prefill": (_I, [_P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, C.c_int32,
                             _P, _P]),
    "qh_gdn_prefill": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                            C.c_int32, C.c_float, _P, _P, C.c_int32, _P]),
    "qh_gdn_chunk_prep": (_I, [_P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                               _P, _P]),
    "qh_gdn_chunked": (_I, [_P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P]),
    "qh_argmax_feed": (_I, [_P, C.c_int32, _I64, _P, _P, _P, C.c_int32, _P, _P, _P, _P]),
    "qh_slm_trace": (_I, [_P, C.c_int32, C.c_char_p]),
    "qh_slm_snapshot": (_I, [_P, _P]),
    "qh_slm_restore": (_I, [_P, _P]),
    "qh_slm_snapshot_free": (None, [_P]),
    "qh_slm_snapshot_bytes": (_I64, [_P]),
    "qh_slm_snapshot_pos": (C.c_int32, [_P]),
    "qh_sampler_defaults": (None, [_P]),
    "qh_rng_seed": (None, [_U64, _P]),
    "qh_sample": (_I, [_P, _P, C.c_int32, _I64, _P, C.c_int32, _P, _P, _P, _P]),
    "qh_sample_feed": (_I, [_P, C.c_int32, _I64, _P, _P, C.c_int32, _P, _P, _P, C.c_int32, _P, _P, _P, _P, _P]),
    "qh_slm_generate_sampled": (_I, [_P, _P, C.c_int32, C.c_int32, C.c_int32, _P, _P, C.c_int32, C.c_int32, _P,
                                     C.c_int32, _P, _P]),
})

class SlmSampler(C.Structure):
    """struct slm_sampler (include/slm.h)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repetition_penalty", C.c_float), ("repetition_window", C.c_int)]


class SlmCtrl(C.Structure):
    """struct slm_ctrl (include/slm.h)."""
    _fields_ = [("tools", C.c_bool), ("think", C.c_bool), ("effort", C.c_char_p), ("debug", C.c_int32),
                ("trace_tokens", C.c_bool), ("dump_layer", C.c_int32)]


SLM_TOKEN_FN = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)

SIGNATURES.update({  # include/slm.h: the reference's slm.h entry points
    "slm_model_load": (_P, [C.c_char_p]),
    "slm_model_unload": (None, [_P]),
    "slm_model_loaded": (C.c_bool, [_P]),
    "slm_model_error": (C.c_char_p, [_P]),
    "slm_ctx_create": (_P, [_P]),
    "slm_ctx_destroy": (None, [_P]),
    "slm_ctx_snapshot": (_P, [_P]),
    "slm_ctx_restore": (None, [_P, _P]),
    "slm_snapshot_free": (None, [_P]),
    "slm_sampler_defaults": (SlmSampler, []),
    "slm_ctrl_defaults": (SlmCtrl, []),
    "slm_ctx_ctrl": (C.POINTER(SlmCtrl), [_P]),
    "slm_generate_ids": (C.c_int, [_P, _P, C.c_int, C.c_int, C.c_int, C.POINTER(SlmSampler), _U64, SLM_TOKEN_FN,
                                   _P]),
    "slm_ctx_tokens": (C.POINTER(C.c_int32), [_P, C.POINTER(C.c_int32)]),
    "slm_vocab_size": (C.c_int, [_P]),
    "slm_eos_id": (C.c_int, [_P]),
    "slm_bos_id": (C.c_int, [_P]),
    "slm_pp_per_sec": (C.c_double, [_P]),
    "slm_tg_per_sec": (C.c_double, [_P]),
    "slm_n_prefill": (C.c_int32, [_P]),
    "slm_n_generated": (C.c_int32, [_P]),
    "qh_gguf_special_tokens": (_I, [C.c_char_p, _P]),
})

SIGNATURES.update({  # include/qh_dp.h
    "qh_dp_unique_id": (_I, [_P]),
    "qh_dp_create": (_I, [_P, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "qh_dp_destroy": (_I, [_P]),
    "qh_dp_rank": (C.c_int32, [_P]),
    "qh_dp_size": (C.c_int32, [_P]),
    "qh_dp_gather_tokens": (_I, [_P, _P, C.c_int32, _P, _P]),
    "qh_dp_wait": (_I, [_P, _P]),
    "qh_dp_max_f64": (_I, [_P, C.POINTER(C.c_double), C.c_int32]),
})

_lib = None


def lib() -> C.CDLL:
    """The loaded libqh200.so with every C-ABI signature declared."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise QHError(-3, "load", f"{LIB_PATH} is missing; run qwen.haiku_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != QH_OK:
        raise QHError(status, where, lib().qh_last_error().decode(errors="replace"))


def row_bytes(gtype: int, k: int) -> int:
    return (k // BLOCK_WEIGHTS[gtype]) * BLOCK_BYTES[gtype]


from . import host  # noqa: E402  (host-side helpers over the bindings)

__all__ = ["lib", "check", "QHError", "MatvecJob", "host", "row_bytes", "SlmSampler", "SlmCtrl", "SLM_TOKEN_FN",
           "F32", "Q8_0", "Q4_K", "Q5_K", "Q6_K", "BLOCK_BYTES", "BLOCK_WEIGHTS"]
