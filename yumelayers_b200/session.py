"""Host-side mirror of the reference's operator API.

``GpuSession`` and ``GPUTensor`` keep the method names, argument meaning and
functional style (each op allocates and returns its output) of the Swift
types they replace -- ``GpuSession`` (GpuTraining.swift:4-151 with the ops of
GpuSessionOps.swift, GpuSessionNormGrad.swift) and ``GPUTensor``
(GPUTensor.swift:9-143) -- so code and tests written against the reference
read the same here.  Every op runs through the C ABI of the CUDA library; a
shape precondition that crashes the reference raises ``YumeError`` here.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import BINARY, UNARY, YumeError, call, lib

_CTX: dict[int, "Context"] = {}


class Context:
    """A ``yl_ctx``: one device, one stream (MetalEngine.swift:6-60)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("yl_ctx_create", device, C.byref(h))
        self.handle = h
        self.device = device

    @classmethod
    def shared(cls, device: int = 0) -> "Context":
        if device not in _CTX:
            _CTX[device] = cls(device)
        return _CTX[device]

    @property
    def stream(self) -> int:
        return lib().yl_ctx_get_stream(self.handle) or 0

    def set_stream(self, stream_ptr: int | None) -> None:
        call("yl_ctx_set_stream", self.handle, C.c_void_p(stream_ptr or 0))

    def set_wait_limit(self, cycles: int) -> None:
        """Bound of the kernels' device-side waits in SM cycles (<= 0: default)."""
        call("yl_ctx_set_wait_limit", self.handle, int(cycles))

    def check_device_errors(self) -> None:
        """Raise (and clear) what a kernel recorded in the device error word."""
        call("yl_ctx_check_device_errors", self.handle)

    def last_kernel(self, which: int = 0) -> str:
        """Template name of the last conv kernel launched: 0 forward / dX, 1 dW."""
        r = lib().yl_ctx_last_kernel(self.handle, int(which))
        return r.decode() if r else ""


class GPUTensor:
    """rows x cols fp32 device tensor (GPUTensor.swift:9-143)."""

    def __init__(self, ctx: Context, rows: int, cols: int | None = None, data=None):
        if data is not None:
            arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
            if cols is None:
                if rows <= 0 or arr.size % rows:
                    raise YumeError(1, f"data of {arr.size} floats does not fill {rows} rows")
                cols = arr.size // rows
            if arr.size != rows * cols:
                raise YumeError(1, f"data of {arr.size} floats for {rows} x {cols}")
        else:
            arr = None
        if cols is None:
            raise YumeError(7, "GPUTensor needs cols or data")
        h = C.c_void_p()
        ptr = arr.ctypes.data_as(C.c_void_p) if arr is not None else None
        call("yl_tensor_create", ctx.handle, int(rows), int(cols), ptr, C.byref(h))
        self.ctx, self.handle, self.rows, self.cols = ctx, h, int(rows), int(cols)

    @property
    def n(self) -> int:
        return self.rows * self.cols

    @property
    def ptr(self) -> int:
        return lib().yl_tensor_data(self.handle)

    def toArray(self) -> np.ndarray:  # noqa: N802 (reference name)
        out = np.empty(self.n, dtype=np.float32)
        call("yl_tensor_download", self.handle, out.ctypes.data_as(C.c_void_p), self.n)
        return out

    def setData(self, data) -> None:  # noqa: N802
        arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
        call("yl_tensor_upload", self.handle, arr.ctypes.data_as(C.c_void_p), arr.size)

    def getValue(self, i: int) -> float:  # noqa: N802
        v = C.c_float()
        call("yl_tensor_get_value", self.handle, int(i), C.byref(v))
        return v.value

    def setValue(self, i: int, v: float) -> None:  # noqa: N802
        call("yl_tensor_set_value", self.handle, int(i), float(v))

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                lib().yl_tensor_release(self.handle)
        except Exception:
            pass


class ScalarBuffer:
    """A one-float device result read after ``end()`` (the reference's shared MTLBuffer)."""

    def __init__(self, ctx: Context):
        self.t = GPUTensor(ctx, 1, 1)

    def value(self) -> float:
        return float(self.t.toArray()[0])


class GpuSession:
    """One recording session (GpuTraining.swift:4-151) with the GpuSession ops."""

    def __init__(self, ctx: Context | None = None):
        self.ctx = ctx or Context.shared(0)
        self.last_gpu_ms = 0.0

    # -- session lifecycle (GpuTraining.swift:17, 123, 140) --
    def begin(self) -> None:
        call("yl_session_begin", self.ctx.handle)

    def commit(self) -> None:
        call("yl_session_commit", self.ctx.handle)

    def end(self, timeout_s: float = 30.0) -> float:
        ms = C.c_double()
        call("yl_session_end", self.ctx.handle, float(timeout_s), C.byref(ms))
        self.last_gpu_ms = ms.value
        return ms.value

    def _new(self, rows: int, cols: int) -> GPUTensor:
        return GPUTensor(self.ctx, rows, cols)

    @staticmethod
    def _same(a: GPUTensor, b: GPUTensor, what: str) -> None:
        if a.n != b.n:
            raise YumeError(1, f"{what}: {a.rows}x{a.cols} and {b.rows}x{b.cols} differ")

    # -- data movement --
    def upload(self, t: GPUTensor, floats) -> None:
        t.setData(floats)

    def copy(self, dst: GPUTensor, src: GPUTensor) -> None:
        self._same(dst, src, "copy")
        call("yl_copy", self.ctx.handle, C.c_void_p(dst.ptr), C.c_void_p(src.ptr), dst.n)

    def zeroFill(self, t: GPUTensor) -> None:  # noqa: N802
        call("yl_zero_fill", self.ctx.handle, C.c_void_p(t.ptr), t.n)

    # -- GEMM and conv primitives --
    def matmul(self, A: GPUTensor, B: GPUTensor, transA=False, transB=False, M=None, N=None,
               K=None) -> GPUTensor:
        m = M if M is not None else (A.cols if transA else A.rows)
        k = K if K is not None else (A.rows if transA else A.cols)
        n = N if N is not None else (B.rows if transB else B.cols)
        out = self._new(m, n)
        call("yl_matmul", self.ctx.handle, A.ptr, B.ptr, out.ptr, m, n, k, int(transA),
             int(transB))
        return out

    def im2col(self, X, ih, iw, ic, kh, kw, stride, pad) -> GPUTensor:
        oh = (ih + 2 * pad - kh) // stride + 1
        ow = (iw + 2 * pad - kw) // stride + 1
        out = self._new(ic * kh * kw, oh * ow)
        call("yl_im2col", self.ctx.handle, X.ptr, out.ptr, ic, ih, iw, kh, kw, stride, pad)
        return out

    def col2im(self, Cm, ic, ih, iw, kh, kw, stride, pad, oh, ow) -> GPUTensor:
        out = self._new(ic, ih * iw)
        call("yl_col2im", self.ctx.handle, Cm.ptr, out.ptr, ic, ih, iw, kh, kw, stride, pad, oh,
             ow)
        return out

    def gradW(self, A, B, oc, kk) -> GPUTensor:  # noqa: N802
        out = self._new(oc, kk)
        call("yl_grad_w", self.ctx.handle, A.ptr, B.ptr, out.ptr, oc, kk, A.cols)
        return out

    def convBackInputS1(self, dOut, W, ic, oc, ih, iw, k, pad) -> GPUTensor:  # noqa: N802,N803
        out = self._new(ic, ih * iw)
        call("yl_conv_back_input_s1", self.ctx.handle, dOut.ptr, W.ptr, out.ptr, ic, oc, ih, iw,
             k, pad)
        return out

    def biasRow(self, A, b) -> GPUTensor:  # noqa: N802
        out = self._new(A.rows, A.cols)
        call("yl_bias_row", self.ctx.handle, A.ptr, b.ptr, out.ptr, A.rows, A.cols)
        return out

    def biasRowGrad(self, G) -> GPUTensor:  # noqa: N802
        out = self._new(G.rows, 1)
        call("yl_bias_row_grad", self.ctx.handle, G.ptr, out.ptr, G.rows, G.cols)
        return out

    def addBias(self, A, bias) -> GPUTensor:  # noqa: N802
        out = self._new(A.rows, A.cols)
        call("yl_add_bias", self.ctx.handle, A.ptr, bias.ptr, out.ptr, A.rows, A.cols)
        return out

    def sumCols(self, A) -> GPUTensor:  # noqa: N802
        out = self._new(1, A.cols)
        call("yl_sum_cols", self.ctx.handle, A.ptr, out.ptr, A.rows, A.cols)
        return out

    # -- normalisation --
    def groupNorm(self, A, groups) -> GPUTensor:  # noqa: N802
        out = self._new(A.rows, A.cols)
        call("yl_group_norm", self.ctx.handle, A.ptr, out.ptr, A.rows, A.cols, groups)
        return out

    def encodeGroupNormGrad(self, x, dy, groups) -> GPUTensor:  # noqa: N802
        out = self._new(x.rows, x.cols)
        call("yl_group_norm_grad", self.ctx.handle, x.ptr, dy.ptr, out.ptr, x.rows, x.cols,
             groups)
        return out

    # -- elementwise --
    def _unary(self, op, A) -> GPUTensor:
        out = self._new(A.rows, A.cols)
        call("yl_unary", self.ctx.handle, UNARY[op], A.ptr, out.ptr, A.n)
        return out

    def _binary(self, op, A, B) -> GPUTensor:
        self._same(A, B, op)
        out = self._new(A.rows, A.cols)
        call("yl_binary", self.ctx.handle, BINARY[op], A.ptr, B.ptr, out.ptr, A.n)
        return out

    def relu(self, A): return self._unary("relu", A)
    def sigmoid(self, A): return self._unary("sigmoid", A)
    def tanh(self, A): return self._unary("tanh", A)
    def tanhGrad(self, A): return self._unary("tanh_grad", A)  # noqa: N802
    def exp(self, A): return self._unary("exp", A)
    def expHalf(self, A): return self._unary("exp_half", A)  # noqa: N802
    def silu(self, A): return self._unary("silu", A)
    def add(self, A, B): return self._binary("add", A, B)
    def sub(self, A, B): return self._binary("sub", A, B)
    def mul(self, A, B): return self._binary("mul", A, B)
    def reluGrad(self, Y, G): return self._binary("relu_grad", Y, G)  # noqa: N802
    def sigmoidGrad(self, Z, G): return self._binary("sigmoid_grad", Z, G)  # noqa: N802
    def siluGrad(self, Z, G): return self._binary("silu_grad", Z, G)  # noqa: N802

    def smul(self, s, A) -> GPUTensor:
        out = self._new(A.rows, A.cols)
        call("yl_smul", self.ctx.handle, float(s), A.ptr, out.ptr, A.n)
        return out

    def addConst(self, A, s) -> GPUTensor:  # noqa: N802
        out = self._new(A.rows, A.cols)
        call("yl_add_const", self.ctx.handle, A.ptr, float(s), out.ptr, A.n)
        return out

    def fma(self, A, B, D) -> GPUTensor:
        if not (A.n == B.n == D.n):
            raise YumeError(1, "fma: sizes must match")
        out = self._new(A.rows, A.cols)
        call("yl_fma", self.ctx.handle, A.ptr, B.ptr, D.ptr, out.ptr, A.n)
        return out

    def addInPlace(self, A, B) -> None:  # noqa: N802
        self._same(A, B, "addInPlace")
        call("yl_add_in_place", self.ctx.handle, A.ptr, B.ptr, A.n)

    # -- resampling --
    def upsample2x(self, X, h, w) -> GPUTensor:
        out = self._new(X.rows, 4 * h * w)
        call("yl_upsample2x", self.ctx.handle, X.ptr, out.ptr, X.rows, h, w)
        return out

    def downsample2x(self, X, h, w) -> GPUTensor:
        out = self._new(X.rows, h * w)
        call("yl_downsample2x", self.ctx.handle, X.ptr, out.ptr, X.rows, h, w)
        return out

    # -- VAE heads --
    def split2(self, X, c, plane):
        if X.n != 2 * c * plane:
            raise YumeError(1, "split2: wrong input shape")
        mu, lv = self._new(c, plane), self._new(c, plane)
        call("yl_split2", self.ctx.handle, X.ptr, mu.ptr, lv.ptr, c, plane)
        return mu, lv

    def merge2(self, A, B, c, plane) -> GPUTensor:
        out = self._new(2 * c, plane)
        call("yl_merge2", self.ctx.handle, A.ptr, B.ptr, out.ptr, c, plane)
        return out

    def randn(self, seed, rows, cols) -> GPUTensor:
        out = self._new(rows, cols)
        call("yl_randn", self.ctx.handle, out.ptr, C.c_uint32(seed & 0xFFFFFFFF), out.n)
        return out

    def kl(self, mu, logvar) -> ScalarBuffer:
        self._same(mu, logvar, "kl")
        buf = ScalarBuffer(self.ctx)
        call("yl_kl_sum", self.ctx.handle, mu.ptr, logvar.ptr, mu.n, buf.t.ptr)
        return buf

    def encodeMSE(self, recon, target) -> ScalarBuffer:  # noqa: N802
        self._same(recon, target, "encodeMSE")
        buf = ScalarBuffer(self.ctx)
        call("yl_mse_sum", self.ctx.handle, recon.ptr, target.ptr, recon.n, buf.t.ptr)
        return buf

    def encodeL1Grad(self, recon, target) -> GPUTensor:  # noqa: N802
        self._same(recon, target, "encodeL1Grad")
        out = self._new(recon.rows, recon.cols)
        call("yl_l1_grad", self.ctx.handle, recon.ptr, target.ptr, out.ptr, recon.n)
        return out

    def vaeGrad(self, dz, mu, logvar, eps, betaN, betaHalfN):  # noqa: N802,N803
        if not (dz.n == mu.n == logvar.n == eps.n):
            raise YumeError(1, "vaeGrad: sizes must match")
        dmu, dlv = self._new(mu.rows, mu.cols), self._new(mu.rows, mu.cols)
        call("yl_vae_grad", self.ctx.handle, dz.ptr, mu.ptr, logvar.ptr, eps.ptr, dmu.ptr,
             dlv.ptr, float(betaN), float(betaHalfN), mu.n)
        return dmu, dlv

    # -- optimiser --
    def adamUpdate(self, param, grad, m, v, t, lr) -> None:  # noqa: N802
        call("yl_adam_update", self.ctx.handle, param.ptr, grad.ptr, m.ptr, v.ptr, param.n,
             int(t), float(lr))
