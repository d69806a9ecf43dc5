"""ctypes binding of libspar_b200.so (the C ABI declared in include/spar_b200.h and
include/spar_cuda_kernels.h).

There is no fallback: if the library is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libspar_b200.so")


class SparCudaStatus(ctypes.Structure):
    _fields_ = [("code", c_int), ("cuda_error", c_int)]


class SparCudaNormSummary(ctypes.Structure):
    _fields_ = [("scale", c_double), ("scaled_sum_squares", c_double),
                ("has_infinity", c_int), ("has_nan", c_int)]


class SparB200TensorSlice(ctypes.Structure):
    _fields_ = [("parameter", c_void_p), ("gradient", c_void_p), ("first_moment", c_void_p),
                ("second_moment", c_void_p), ("count", c_uint64)]


class SparB200Gemm(ctypes.Structure):
    _fields_ = [
        ("m", c_uint64), ("n", c_uint64), ("k", c_uint64), ("batch", c_uint64 * 2),
        ("a", c_void_p), ("lda", c_uint64), ("a_batch_stride", c_uint64 * 2), ("a_transposed", c_int),
        ("b", c_void_p), ("ldb", c_uint64), ("b_batch_stride", c_uint64 * 2), ("b_transposed", c_int),
        ("c", c_void_p), ("ldc", c_uint64), ("c_batch_stride", c_uint64 * 2),
        ("alpha", c_float), ("accumulate", c_int), ("epilogue", c_int), ("bias", c_void_p),
        ("aux", c_void_p), ("ldaux", c_uint64), ("precision", c_int), ("causal", c_int),
        ("round_output", c_int), ("rope_table", c_void_p), ("rope_seq", c_uint64),
        ("rope_dim", c_uint64), ("rope_cols", c_uint64), ("column_partials", c_void_p),
    ]


class SparB200Checkpoint(ctypes.Structure):
    _fields_ = [("global_step", c_uint64), ("tokens_seen", c_uint64), ("rng_state", c_uint64),
                ("learning_rate", c_double), ("adam_step", c_uint64)]


class SparB200LMConfig(ctypes.Structure):
    _fields_ = [
        ("vocab_size", c_uint64), ("model_dim", c_uint64), ("hidden_dim", c_uint64),
        ("num_layers", c_uint64), ("num_heads", c_uint64), ("sequence_length", c_uint64),
        ("micro_batch", c_uint64), ("norm_epsilon", c_double), ("rope_theta", c_double),
        ("use_rope", c_int), ("precision", c_int),
        ("beta1", c_double), ("beta2", c_double), ("adam_epsilon", c_double),
        ("weight_decay", c_double), ("max_grad_norm", c_double),
        ("family", c_int), ("qk_norm", c_int), ("num_kv_heads", c_uint64),
        ("qk_norm_epsilon", c_double),
    ]


S = SparCudaStatus
p, u64, i, d, f = c_void_p, c_uint64, c_int, c_double, c_float

SIGNATURES = {
    # ---- new asynchronous entry points (include/spar_b200.h)
    "spar_b200_layernorm_forward": (S, [p, p, p, p, p, p, u64, u64, d, i, p]),
    "spar_b200_layernorm_backward": (S, [p, p, p, p, p, p, p, p, u64, u64, i, i, i, p]),
    "spar_b200_layernorm_backward_noalloc": (S, [p, p, p, p, p, p, p, p, u64, u64, i, i, i, p]),
    "spar_b200_rmsnorm_forward": (S, [p, p, p, p, u64, u64, d, i, p]),
    "spar_b200_rmsnorm_backward": (S, [p, p, p, p, p, p, u64, u64, i, i, i, p]),
    "spar_b200_head_rmsnorm_forward": (S, [p, p, u64, u64, u64, u64, p, p, d, i, p]),
    "spar_b200_head_rmsnorm_backward": (S, [p, p, p, p, u64, u64, u64, u64, p, p, i, i, p]),
    "spar_b200_swiglu_forward": (S, [p, u64, p, u64, p, u64, u64, u64, i, p]),
    "spar_b200_swiglu_backward": (S, [p, u64, p, u64, p, u64, p, u64, p, u64, u64, u64, i, p]),
    "spar_b200_gelu_forward": (S, [p, p, u64, i, p]),
    "spar_b200_gelu_backward": (S, [p, p, p, u64, i, p]),
    "spar_b200_causal_softmax_forward": (S, [p, p, u64, u64, u64, f, u64, i, p]),
    "spar_b200_causal_softmax_backward": (S, [p, p, p, u64, u64, u64, f, u64, i, p]),
    "spar_b200_cross_entropy_forward_backward": (S, [p, p, p, p, u64, u64, u64, u64, f, p, i, p]),
    "spar_b200_sum": (S, [p, p, u64, i, p]),
    "spar_b200_grad_norm_squared": (S, [p, POINTER(SparB200TensorSlice), u64, i, p]),
    "spar_b200_adamw_clipped": (S, [POINTER(SparB200TensorSlice), u64, p, d, d, d, d, d, d, u64,
                                    p, i, p]),
    "spar_b200_embedding_forward": (S, [p, p, p, u64, u64, u64, p, i, p]),
    "spar_b200_embedding_backward_scratch_bytes": (u64, [u64, u64]),
    "spar_b200_embedding_backward": (S, [p, p, p, u64, u64, u64, p, i, p]),
    "spar_b200_column_sum": (S, [p, p, u64, u64, u64, i, i, p]),
    "spar_b200_rope_table": (S, [p, u64, u64, d, u64, i, p]),
    "spar_b200_rope_apply": (S, [p, p, u64, u64, u64, u64, u64, i, i, p]),
    "spar_b200_gemm": (S, [POINTER(SparB200Gemm), i, p]),
    "spar_b200_gemm_error": (c_int, [i, i]),
    "spar_b200_matmul": (S, [p, p, p, u64, u64, u64, u64, i, i, i, p]),
    "spar_b200_attention_forward": (S, [p, p, p, p, u64, u64, u64, u64, i, p]),
    "spar_b200_attention_backward": (S, [p, p, p, p, p, p, p, u64, u64, u64, u64, p, i, p]),
    "spar_b200_attention_forward_gqa": (S, [p, p, p, p, u64, u64, u64, u64, u64, i, p]),
    "spar_b200_attention_backward_gqa": (S, [p, p, p, p, p, p, p, u64, u64, u64, u64, u64, p, i,
                                             p]),
    "spar_b200_attention_error": (c_int, [i, i]),
    "spar_b200_set_wait_error": (c_int, [i, i, i]),
    "spar_b200_lm_create": (S, [POINTER(SparB200LMConfig), i, POINTER(c_void_p)]),
    "spar_b200_lm_destroy": (None, [p]),
    "spar_b200_lm_parameter_count": (u64, [p]),
    "spar_b200_lm_flat_size": (u64, [p]),
    "spar_b200_lm_flat_buffer": (c_void_p, [p, i]),
    "spar_b200_lm_parameter_info": (S, [p, u64, c_char_p, u64, POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_parameter_copy": (S, [p, u64, i, i, p]),
    "spar_b200_lm_init_normal": (S, [p, u64, d, p]),
    "spar_b200_lm_zero_grad": (S, [p, p]),
    "spar_b200_lm_forward_backward": (S, [p, p, u64, f, i, p]),
    "spar_b200_lm_optimizer_step": (S, [p, d, u64, p]),
    "spar_b200_lm_train_step": (S, [p, p, i, u64, d, u64, POINTER(c_float), POINTER(c_double),
                                    POINTER(c_int32), p]),
    "spar_b200_lm_set_comm": (S, [p, p, i]),
    "spar_b200_lm_gather": (S, [p, i, p]),
    "spar_b200_batches_create": (S, [p, u64, u64, u64, u64, i, u64, i, i, i, i,
                                     POINTER(c_void_p)]),
    "spar_b200_batches_next": (S, [p, p, POINTER(c_uint64), POINTER(c_uint64), p]),
    "spar_b200_batches_next_epoch": (S, [p]),
    "spar_b200_batches_state": (S, [p, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_batches_set_state": (S, [p, u64, u64]),
    "spar_b200_batches_destroy": (None, [p]),
    "spar_b200_split_documents": (S, [u64, u64, u64, p]),
    "spar_b200_batch_windows": (S, [u64, u64, u64, u64, i, u64, i, u64, u64, i, i, p,
                                    POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_save_checkpoint": (S, [p, c_char_p, POINTER(SparB200Checkpoint)]),
    "spar_b200_lm_load_checkpoint": (S, [p, c_char_p, POINTER(SparB200Checkpoint)]),
    "spar_b200_checkpoint_write": (S, [c_char_p, POINTER(SparB200LMConfig),
                                       POINTER(SparB200Checkpoint), p, p, p]),
    "spar_b200_checkpoint_read": (S, [c_char_p, POINTER(SparB200LMConfig),
                                      POINTER(SparB200Checkpoint), p, p, p]),
    "spar_b200_lm_layout": (S, [p, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_layout_tensor": (S, [p, u64, c_char_p, u64, POINTER(c_uint64), POINTER(c_uint64),
                                       POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_layout_bucket": (S, [p, u64, POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_layout_shard": (S, [p, u64, i, i, POINTER(c_uint64), POINTER(c_uint64),
                                      POINTER(c_uint64), POINTER(c_uint64)]),
    "spar_b200_lm_read_losses": (S, [p, p, u64]),
    "spar_b200_warmup_cosine": (d, [d, d, u64, u64, u64]),
    "spar_b200_lm_profile": (S, [p, i]),
    "spar_b200_lm_profile_read": (S, [p, POINTER(c_double), POINTER(c_double), POINTER(c_uint64),
                                      POINTER(c_uint64)]),
    "spar_b200_comm_unique_id": (S, [c_char_p, u64]),
    "spar_b200_comm_init": (S, [c_char_p, i, i, i, POINTER(c_void_p)]),
    "spar_b200_comm_allreduce_sum": (S, [p, p, u64, p]),
    "spar_b200_comm_check": (S, [p]),
    "spar_b200_comm_destroy": (S, [p, i]),
    "spar_b200_comm_set_timeout": (S, [p, d]),
    "spar_b200_comm_wait": (S, [p, p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libspar_b200.so once and attaches argument/return types."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m spar_b200.build` "
            "(spar_b200 has no CPU fallback)")
    import torch  # noqa: F401  (loads the CUDA runtime/NCCL the library shares with torch)
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    for name, (res, args) in EXTRA_SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is not None:
            fn.restype = res
            fn.argtypes = args
    _lib = lib
    return lib


# Drop-in ABI of the reference backend (include/spar_cuda_kernels.h), synchronous.
EXTRA_SIGNATURES = {
    "spar_cuda_launch_binary": (S, [p, p, p, u64, i, i, i]),
    "spar_cuda_launch_scalar": (S, [p, p, u64, i, i, d, i]),
    "spar_cuda_launch_unary": (S, [p, p, u64, i, i, i]),
    "spar_cuda_launch_reduction": (S, [p, p, u64, i, i, i]),
    "spar_cuda_launch_row_reduction": (S, [p, p, u64, u64, i, i, i]),
    "spar_cuda_launch_probability_forward": (S, [p, p, p, u64, u64, u64, i, i, i]),
    "spar_cuda_launch_probability_backward": (S, [p, p, p, p, u64, u64, u64, i, i, i]),
    "spar_cuda_launch_validate_embedding_indices": (S, [p, p, u64, u64, i, i]),
    "spar_cuda_launch_embedding_forward": (S, [p, p, p, p, u64, u64, u64, i, i, i]),
    "spar_cuda_launch_embedding_backward": (S, [p, p, p, u64, u64, i, i, i]),
    "spar_cuda_launch_rope": (S, [p, p, u64, u64, u64, u64, d, i, i, i]),
    "spar_cuda_launch_causal_mask": (S, [p, u64, i, i]),
    "spar_cuda_launch_fill_from_scalar": (S, [p, p, u64, i, d, i]),
    "spar_cuda_launch_add_in_place": (S, [p, p, u64, i, i]),
    "spar_cuda_launch_strided_copy": (S, [p, p, u64, POINTER(c_uint64), POINTER(c_uint64), u64,
                                          u64, u64, i]),
    "spar_cuda_launch_broadcast_reduce": (S, [p, p, u64, POINTER(c_uint64), u64,
                                              POINTER(c_uint64), POINTER(c_uint64), u64, i, i]),
    "spar_cuda_validate_targets": (S, [p, p, u64, u64, i, i]),
    "spar_cuda_launch_nll_forward": (S, [p, p, p, u64, u64, u64, i, i, i, i]),
    "spar_cuda_launch_nll_backward": (S, [p, p, p, u64, u64, u64, i, i, i, i]),
    "spar_cuda_gradient_norm_summary": (S, [POINTER(SparCudaNormSummary), p, u64, i, i]),
    "spar_cuda_launch_scale_in_place": (S, [p, u64, i, d, i]),
    "spar_cuda_launch_adamw": (S, [p, p, p, p, u64, i, d, d, d, d, d, d, d, i]),
    "spar_cuda_error_string": (c_char_p, [c_int]),
    "spar_b200_version": (c_char_p, []),
}


class SparError(RuntimeError):
    """A non-zero SparCudaStatus, with the reference's code meaning (1 invalid, 2 CUDA)."""

    def __init__(self, name: str, status: SparCudaStatus):
        self.code = status.code
        self.cuda_error = status.cuda_error
        kind = {1: "invalid argument", 2: "CUDA runtime error"}.get(status.code, "error")
        super().__init__(f"{name} failed: {kind} (code {status.code}, cuda error {status.cuda_error})")


def check(name: str, status: SparCudaStatus) -> None:
    if status.code != 0:
        raise SparError(name, status)


def call(name: str, *args):
    """Calls a status-returning entry point and raises SparError on failure."""
    fn = getattr(load(), name)
    status = fn(*args)
    check(name, status)
    return status


def exported_symbols() -> list[str]:
    return list(SIGNATURES) + list(EXTRA_SIGNATURES)


_ = (c_int32,)
