"""ctypes binding of ``include/yume_c.h`` (the backend's C ABI).

Loading fails loudly: there is no CPU or PyTorch fallback behind these
symbols.  Build the library first with ``python -m yumelayers_b200.build``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libyumecuda.so"

YL_OK = 0
STATUS_NAMES = {
    0: "YL_OK", 1: "YL_ERR_SHAPE", 2: "YL_ERR_OOM", 3: "YL_ERR_TIMEOUT", 4: "YL_ERR_CUDA",
    5: "YL_ERR_NCCL", 6: "YL_ERR_DEVICE_ASSERT", 7: "YL_ERR_INVALID", 8: "YL_ERR_UNSUPPORTED",
}
LAYOUT_NCHW, LAYOUT_NHWC = 0, 1
UNARY = {"relu": 0, "sigmoid": 1, "tanh": 2, "tanh_grad": 3, "exp": 4, "exp_half": 5, "silu": 6}
BINARY = {"add": 0, "sub": 1, "mul": 2, "relu_grad": 3, "sigmoid_grad": 4, "silu_grad": 5}


class YumeError(RuntimeError):
    """A non-OK yl_status, with the library's thread-local message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class ConvDesc(C.Structure):
    """``yl_conv_desc``."""
    _fields_ = [(n, C.c_int) for n in ("n", "c", "h", "w", "oc", "k", "stride", "pad", "up",
                                        "up_h", "up_w", "layout")]


class AdamTensor(C.Structure):
    """``yl_adam_tensor``."""
    _fields_ = [("param", C.c_void_p), ("grad", C.c_void_p), ("m", C.c_void_p),
                ("v", C.c_void_p), ("n", C.c_longlong)]


class TrainerConfig(C.Structure):
    """``yl_trainer_config``."""
    _fields_ = [("batch", C.c_int), ("height", C.c_int), ("width", C.c_int),
                ("seed", C.c_uint64), ("lr_vae", C.c_float), ("lr_motion", C.c_float),
                ("beta_kl", C.c_float), ("clip_max_norm", C.c_float), ("train_vae", C.c_int),
                ("train_motion", C.c_int), ("bucket_bytes", C.c_size_t), ("profile", C.c_int)]


KERNEL_CLASSES = 6


class KernelStats(C.Structure):
    """``yl_kernel_stats``: conv fprop, conv dgrad, conv wgrad, GN fwd, GN bwd, and the
    dominant launch type (3x3 128->128 fprop/dX at the frame resolution, also in 0/1)."""
    _fields_ = [("ms", C.c_double * KERNEL_CLASSES), ("flops", C.c_double * KERNEL_CLASSES),
                ("bytes", C.c_double * KERNEL_CLASSES), ("launches", C.c_int * KERNEL_CLASSES),
                ("exec_flops", C.c_double * KERNEL_CLASSES)]


P = C.c_void_p
I = C.c_int
F = C.c_float
D = C.c_double
SZ = C.c_size_t
U32 = C.c_uint32
I64 = C.c_int64
LL = C.c_longlong

# name -> argument types (every function returns yl_status unless listed in _RET)
SIGNATURES: dict[str, list] = {
    "yl_ctx_create": [I, C.POINTER(P)],
    "yl_ctx_destroy": [P],
    "yl_ctx_set_stream": [P, P],
    "yl_ctx_get_stream": [P],
    "yl_session_begin": [P],
    "yl_session_commit": [P],
    "yl_session_end": [P, D, C.POINTER(D)],
    "yl_ctx_check_device_errors": [P],
    "yl_tensor_create": [P, I, I, P, C.POINTER(P)],
    "yl_tensor_release": [P],
    "yl_tensor_data": [P],
    "yl_tensor_rows": [P],
    "yl_tensor_cols": [P],
    "yl_tensor_upload": [P, P, SZ],
    "yl_tensor_download": [P, P, SZ],
    "yl_tensor_get_value": [P, SZ, C.POINTER(F)],
    "yl_tensor_set_value": [P, SZ, F],
    "yl_copy": [P, P, P, SZ],
    "yl_zero_fill": [P, P, SZ],
    "yl_memcpy_htod": [P, P, P, SZ],
    "yl_memcpy_dtoh": [P, P, P, SZ],
    "yl_matmul": [P, P, P, P, I, I, I, I, I],
    "yl_im2col": [P, P, P, I, I, I, I, I, I, I],
    "yl_col2im": [P, P, P, I, I, I, I, I, I, I, I, I],
    "yl_grad_w": [P, P, P, P, I, I, I],
    "yl_conv_back_input_s1": [P, P, P, P, I, I, I, I, I, I],
    "yl_bias_row": [P, P, P, P, I, I],
    "yl_bias_row_grad": [P, P, P, I, I],
    "yl_add_bias": [P, P, P, P, I, I],
    "yl_sum_cols": [P, P, P, I, I],
    "yl_group_norm": [P, P, P, I, I, I],
    "yl_group_norm_grad": [P, P, P, P, I, I, I],
    "yl_unary": [P, I, P, P, SZ],
    "yl_binary": [P, I, P, P, P, SZ],
    "yl_smul": [P, F, P, P, SZ],
    "yl_add_const": [P, P, F, P, SZ],
    "yl_fma": [P, P, P, P, P, SZ],
    "yl_add_in_place": [P, P, P, SZ],
    "yl_upsample2x": [P, P, P, I, I, I],
    "yl_downsample2x": [P, P, P, I, I, I],
    "yl_split2": [P, P, P, P, I, I],
    "yl_merge2": [P, P, P, P, I, I],
    "yl_randn": [P, P, U32, SZ],
    "yl_mse_sum": [P, P, P, SZ, P],
    "yl_kl_sum": [P, P, P, SZ, P],
    "yl_l1_grad": [P, P, P, P, SZ],
    "yl_vae_grad": [P, P, P, P, P, P, P, F, F, SZ],
    "yl_adam_update": [P, P, P, P, P, SZ, I, F],
    "yl_conv2d_out_shape": [C.POINTER(ConvDesc), C.POINTER(I), C.POINTER(I)],
    "yl_conv2d_fwd": [P, C.POINTER(ConvDesc), P, P, P, P, P],
    "yl_conv2d_bwd_data": [P, C.POINTER(ConvDesc), P, P, P],
    "yl_conv2d_bwd_filter": [P, C.POINTER(ConvDesc), P, P, P, P],
    "yl_conv_transpose2d_fwd": [P, C.POINTER(ConvDesc), P, P, P, P],
    "yl_conv_transpose2d_bwd_data": [P, C.POINTER(ConvDesc), P, P, P],
    "yl_conv_transpose2d_bwd_filter": [P, C.POINTER(ConvDesc), P, P, P, P],
    "yl_groupnorm_silu_fwd": [P, P, I, I, I, I, I, I, F, I, P, P, I, P, P, P],
    "yl_groupnorm_silu_bwd": [P, P, P, I, I, I, I, I, I, F, I, P, P, I, P, P, P, P, P, P],
    "yl_groupnorm_silu_fwd_noalloc": [P, P, I, I, I, I, I, F, I, P, P, I, P, P, P],
    "yl_linear_fwd": [P, P, P, P, P, I, I, I],
    "yl_linear_bwd": [P, P, P, P, P, P, P, I, I, I],
    "yl_timestep_embedding": [P, P, I, I, I, P],
    "yl_adam_multi": [P, C.POINTER(AdamTensor), I, F, F, F, F, I, F, F, I, P],
    "yl_vae_latent_head_fwd": [P, P, I, I, I, I, I, I64, P],
    "yl_vae_latent_head_bwd": [P, P, P, I, I, I, I, I, I64, F, P],
    "yl_loss_l1_kl": [P, P, P, SZ, P, I, I, I, I, I, F, P, P],
    "yl_comm_get_unique_id": [P],
    "yl_comm_init": [P, P, I, I, C.POINTER(P)],
    "yl_comm_destroy": [P],
    "yl_comm_abort": [P],
    "yl_allreduce_sum": [P, P, SZ, P],
    "yl_trainer_create": [P, C.POINTER(TrainerConfig), P, C.POINTER(P)],
    "yl_trainer_destroy": [P],
    "yl_trainer_step": [P, P, P, P],
    "yl_trainer_step_host": [P, P, P, P],
    "yl_trainer_set_config": [P, C.POINTER(TrainerConfig)],
    "yl_trainer_param_count": [P, I, C.POINTER(SZ)],
    "yl_trainer_buffer": [P, I, I, C.POINTER(P)],
    "yl_trainer_param_entry": [P, I, I, C.c_char_p, SZ, C.POINTER(SZ), C.POINTER(I)],
    "yl_trainer_prepare_weights": [P],
    "yl_trainer_kernel_stats": [P, C.POINTER(KernelStats), I],
    "yl_trainer_activation_bytes": [P, C.POINTER(SZ)],
}
class TemplateStats(C.Structure):
    """``yl_template_stats``."""
    _fields_ = [("name", C.c_char * 96), ("ms", C.c_double), ("flops", C.c_double),
                ("exec_flops", C.c_double), ("launches", C.c_int)]


SIGNATURES["yl_trainer_template_stats"] = [P, C.POINTER(TemplateStats), I, C.POINTER(I)]
SIGNATURES["yl_trainer_comm_stats"] = [P, C.POINTER(D), C.POINTER(I), I]
SIGNATURES["yl_comm_init_timeout"] = [P, P, I, I, D, C.POINTER(P)]
SIGNATURES["yl_ctx_set_wait_limit"] = [P, C.c_longlong]
SIGNATURES["yl_ctx_last_kernel"] = [P, I]
SIGNATURES["yl_debug_wait_probe"] = [P]
SIGNATURES["yl_debug_spin"] = [P, D]
_RET = {"yl_last_error_message": C.c_char_p, "yl_version": C.c_char_p,
        "yl_kernel_launch_count": C.c_ulonglong, "yl_ctx_last_kernel": C.c_char_p,
        "yl_ctx_get_stream": P, "yl_tensor_data": P, "yl_tensor_rows": I, "yl_tensor_cols": I}
NON_STATUS = set(_RET)

_lib = None


def lib() -> C.CDLL:
    """Load (once) the in-tree CUDA library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m yumelayers_b200.build`. "
            "There is no CPU fallback for the backend's operators.")
    L = C.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = _RET.get(name, I)
    for name, res in _RET.items():
        getattr(L, name).restype = res
    L.yl_last_error_message.argtypes = []
    L.yl_version.argtypes = []
    L.yl_kernel_launch_count.argtypes = []
    _lib = L
    return L


def check(status: int) -> None:
    """Raise YumeError for a non-OK yl_status."""
    if status != YL_OK:
        msg = lib().yl_last_error_message()
        raise YumeError(status, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    """Call a status-returning C entry point and raise on failure."""
    check(getattr(lib(), name)(*args))


class ConvProfile(C.Structure):
    """``yl_conv_profile``."""
    _fields_ = [("fprop_ms", C.c_double), ("dgrad_ms", C.c_double), ("wgrad_ms", C.c_double),
                ("flops", C.c_double), ("wgrad_splits", C.c_int)]


SIGNATURES["yl_profile_conv"] = [P, I, I, I, I, I, I, I, I, I, C.POINTER(ConvProfile)]
SIGNATURES["yl_profile_groupnorm"] = [P, I, I, I, I, I, C.POINTER(D), C.POINTER(D), C.POINTER(D)]
SIGNATURES["yl_trainer_interpolate"] = [P, P, P, P, I, I, P]
SIGNATURES["yl_interpolation_plan"] = [D, I, I, P, C.POINTER(I)]
SIGNATURES["yl_trainer_get_step"] = [P, C.POINTER(C.c_int64)]
SIGNATURES["yl_trainer_set_step"] = [P, C.c_int64]
SIGNATURES["yl_sobel_edge_loss"] = [P, P, P, I, I, I, I, I, P, P]
SIGNATURES["yl_layered_loss"] = [P, P, P, P, I, LL, F, F, P, P]
SIGNATURES["yl_layered_compose"] = [P, P, I, LL, P]
SIGNATURES["yl_profile_adam"] = [P, C.c_longlong, I, I, C.POINTER(D)]
SIGNATURES["yl_profile_layered"] = [P, I, C.c_longlong, I, C.POINTER(D)]
