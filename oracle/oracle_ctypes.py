"""ctypes loader of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

The oracle restates the reference's hot-path arithmetic in C; tests compare
the CUDA backend against it.  Nothing in the product imports this module.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_SO = ORACLE_DIR / "liboracle.so"

P = C.c_void_p
I = C.c_int
F = C.c_float
D = C.c_double
L = C.c_longlong

_SIGS = {
    "orc_matmul": ([P, P, P, I, I, I, I, I], None),
    "orc_im2col": ([P, P, I, I, I, I, I, I, I], None),
    "orc_col2im": ([P, P, I, I, I, I, I, I, I, I, I], None),
    "orc_conv_back_input_s1": ([P, P, P, I, I, I, I, I, I, I], None),
    "orc_gradw": ([P, P, P, I, I, I], None),
    "orc_bias_row": ([P, P, P, I, I], None),
    "orc_bias_row_grad": ([P, P, I, I], None),
    "orc_add_bias": ([P, P, P, I, I], None),
    "orc_sum_cols": ([P, P, I, I], None),
    "orc_upsample2x": ([P, P, I, I, I], None),
    "orc_downsample2x": ([P, P, I, I, I], None),
    "orc_groupnorm_ref": ([P, P, I, I, I], None),
    "orc_groupnorm_grad_ref": ([P, P, P, I, I, I], None),
    "orc_unary": ([I, P, P, I], None),
    "orc_binary": ([I, P, P, P, I], None),
    "orc_smul": ([P, P, F, I], None),
    "orc_addconst": ([P, P, F, I], None),
    "orc_fma": ([P, P, P, P, I], None),
    "orc_mse_sum": ([P, P, I], D),
    "orc_kl_sum": ([P, P, I], D),
    "orc_l1grad": ([P, P, P, F, I], None),
    "orc_vae_grad": ([P, P, P, P, P, P, F, F, I], None),
    "orc_split2": ([P, P, P, I, I], None),
    "orc_merge2": ([P, P, P, I, I], None),
    "orc_randn": ([P, C.c_uint32, I], None),
    "orc_yume_hash": ([C.c_uint32], C.c_uint32),
    "orc_splitmix64_next": ([C.POINTER(C.c_uint64)], C.c_uint64),
    "orc_training_noise_seed": ([C.c_int64, C.c_int64], C.c_uint32),
    "orc_adam": ([P, P, P, P, I, I, F, F, F, F], None),
    "orc_sanitize_grads": ([P, C.c_long, F, F, C.POINTER(C.c_long)], F),
    "orc_motion_time_embedding": ([D, I, P], None),
    "orc_time_embedding_int": ([I, I, P], None),
    "orc_timestep_embedding_torch": ([P, I, I, F, P], None),
    "orc_conv2d_fwd": ([P, I, I, I, I, P, P, I, I, I, I, I, I, I, P, P, P], None),
    "orc_conv2d_bwd": ([P, I, I, I, I, P, I, I, I, I, I, I, I, P, P, P, P, P], None),
    "orc_gn_silu_fwd": ([P, I, I, I, I, F, P, P, I, P, P, P], None),
    "orc_gn_silu_bwd": ([P, P, I, I, I, I, F, P, P, I, P, P, P, P], None),
    "orc_linear_fwd": ([P, P, P, P, I, I, I, I], None),
    "orc_linear_bwd": ([P, P, P, P, P, P, I, I, I], None),
    "orc_l1_kl_loss": ([P, P, C.c_long, P, P, C.c_long, F, P], D),
    "orc_sobel_luma": ([P, I, I, P], None),
    "orc_sobel_edge_loss": ([P, P, I, I], D),
    "orc_sobel_edge_grad": ([P, P, I, I, P], None),
    "orc_layered_compose": ([P, L, P], None),
    "orc_layered_loss": ([P, P, P, L, F, F], D),
    "orc_layered_grad": ([P, P, P, L, F, F, P], None),
    "orc_num_threads": ([], I),
    "orc_set_num_threads": ([I], None),
}


def ptr(a):
    """Pointer to a contiguous float32/other numpy array (None passes NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _keep_freed_memory():
    """Full-resolution oracle passes allocate and free arrays of hundreds of
    MB; glibc would hand each one back to the kernel (mmap / trim) and fault
    its pages in again on the next allocation.  Serve them from the heap and
    keep freed memory instead (glibc mallopt M_MMAP_MAX = 0, M_TRIM_THRESHOLD
    = 2^62); a no-op where libc has no mallopt."""
    try:
        libc = C.CDLL("libc.so.6")
        libc.mallopt(-4, 0)
        libc.mallopt(-1, C.c_int(2**31 - 1))
    except (OSError, AttributeError):
        pass


def load_oracle():
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(ORACLE_DIR)], check=True, capture_output=True)
    _keep_freed_memory()
    L = C.CDLL(str(ORACLE_SO))
    for name, (args, res) in _SIGS.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


# ---- convenience wrappers returning numpy arrays ----

def conv2d_fwd(L, x, w, b=None, stride=1, pad=1, up=False, up_hw=None, bias2d=None,
               residual=None):
    x, w = f32(x), f32(w)
    n, c, h, wd = x.shape
    oc, k = w.shape[0], w.shape[-1]
    hin, win = (up_hw if up_hw else (2 * h, 2 * wd)) if up else (h, wd)
    oh, ow = (hin + 2 * pad - k) // stride + 1, (win + 2 * pad - k) // stride + 1
    y = np.empty((n, oc, oh, ow), np.float32)  # every element is written
    L.orc_conv2d_fwd(ptr(x), n, c, h, wd, ptr(w), ptr(f32(b) if b is not None else None), oc, k,
                     stride, pad, int(up), hin, win,
                     ptr(f32(bias2d) if bias2d is not None else None),
                     ptr(f32(residual) if residual is not None else None), ptr(y))
    return y


def conv2d_bwd(L, x, w, dy, stride=1, pad=1, up=False, up_hw=None):
    x, w, dy = f32(x), f32(w), f32(dy)
    n, c, h, wd = x.shape
    oc, k = w.shape[0], w.shape[-1]
    hin, win = (up_hw if up_hw else (2 * h, 2 * wd)) if up else (h, wd)
    dx = np.empty_like(x)  # dx, dw, db and dbi are overwritten whole
    dw = np.empty_like(w)
    db = np.empty(oc, np.float32)
    dbi = np.empty((n, oc), np.float32)
    L.orc_conv2d_bwd(ptr(x), n, c, h, wd, ptr(w), oc, k, stride, pad, int(up), hin, win, ptr(dy),
                     ptr(dx), ptr(dw), ptr(db), ptr(dbi))
    return dx, dw, db, dbi


def gn_silu_fwd(L, x, groups, eps, gamma=None, beta=None, silu=True):
    x = f32(x)
    n, c, h, w = x.shape
    y = np.empty_like(x)  # every element is written
    m = np.empty(n * groups, np.float32)
    r = np.empty(n * groups, np.float32)
    L.orc_gn_silu_fwd(ptr(x), n, c, h * w, groups, eps, ptr(f32(gamma) if gamma is not None else None),
                      ptr(f32(beta) if beta is not None else None), int(silu), ptr(y), ptr(m), ptr(r))
    return y, m, r


def gn_silu_bwd(L, x, dy, groups, eps, gamma=None, beta=None, silu=True, addend=None):
    x, dy = f32(x), f32(dy)
    n, c, h, w = x.shape
    dx = np.empty_like(x)  # every element is written
    dg = np.empty(c, np.float32)
    db = np.empty(c, np.float32)
    L.orc_gn_silu_bwd(ptr(x), ptr(dy), n, c, h * w, groups, eps,
                      ptr(f32(gamma) if gamma is not None else None),
                      ptr(f32(beta) if beta is not None else None), int(silu),
                      ptr(f32(addend) if addend is not None else None), ptr(dx), ptr(dg), ptr(db))
    return dx, dg, db


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
