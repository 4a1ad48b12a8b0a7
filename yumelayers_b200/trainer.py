"""Python driver of the joint VAE + motion-net training step (``yl_trainer_*``).

The step itself runs in the CUDA library; this module only creates the
context, optionally joins the data-parallel group (one process per GPU:
``torch.distributed`` carries the NCCL unique id and the barriers, the
library's own NCCL communicator carries the gradients), and moves buffers.
"""
from __future__ import annotations

import ctypes as C
import weakref
from dataclasses import dataclass

import numpy as np

from ._lib import KernelStats, TemplateStats, TrainerConfig, YumeError, call, lib
from .session import Context


CLASS_NAMES = ["conv_fprop", "conv_dgrad", "conv_wgrad", "gn_silu_fwd", "gn_silu_bwd",
               "conv_3x3_128_frame"]


def _bind() -> C.CDLL:
    return lib()


def default_config(batch=8, height=480, width=856, seed=0, **kw) -> TrainerConfig:
    cfg = TrainerConfig(batch=batch, height=height, width=width, seed=seed, lr_vae=2e-4,
                        lr_motion=2e-4, beta_kl=1e-6, clip_max_norm=0.0, train_vae=1,
                        train_motion=1, bucket_bytes=0, profile=0)
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cfg


@dataclass
class ParamEntry:
    name: str
    offset: int
    shape: tuple


class Comm:
    """The library's NCCL communicator for one rank."""

    def __init__(self, ctx: Context, id_bytes: bytes, rank: int, world: int,
                 timeout_s: float = 300.0):
        _bind()
        h = C.c_void_p()
        buf = (C.c_uint8 * 128).from_buffer_copy(id_bytes)
        call("yl_comm_init_timeout", ctx.handle, buf, rank, world, float(timeout_s), C.byref(h))
        self._users = []  # trainers borrowing this communicator (weak references)
        self.handle, self.rank, self.world = h, rank, world

    @staticmethod
    def unique_id() -> bytes:
        _bind()
        buf = (C.c_uint8 * 128)()
        call("yl_comm_get_unique_id", buf)
        return bytes(buf)

    def abort(self) -> None:
        call("yl_comm_abort", self.handle)

    def close(self) -> None:
        """Destroys the communicator; trainers still using it are closed first
        (a trainer must not outlive the communicator it borrows)."""
        for ref in getattr(self, "_users", []):
            t = ref()
            if t is not None:
                t.close()
        if self.handle:
            call("yl_comm_destroy", self.handle)
            self.handle = None


def share_unique_id(rank: int, get_id, broadcast) -> bytes:
    """Rank 0 creates the NCCL id; `broadcast(list)` distributes it (torch.distributed
    broadcast_object_list in production, a fake in the CPU tests)."""
    obj = [get_id() if rank == 0 else None]
    broadcast(obj)
    return obj[0]


def shard_batch(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Weak-scaling split of a global batch: [start, stop) of this rank's samples."""
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} is not divisible by {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def max_over_ranks(x: float, device: str = "cpu") -> float:
    """The maximum of a per-rank scalar (a timed duration) over the default
    torch.distributed group; the scalar itself when there is no group."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Trainer:
    """One rank's joint trainer (``yl_trainer``)."""

    def __init__(self, cfg: TrainerConfig, ctx: Context | None = None, comm: Comm | None = None):
        self.L = _bind()
        self.ctx = ctx or Context.shared(0)
        self.cfg = cfg
        self.comm = comm
        h = C.c_void_p()
        call("yl_trainer_create", self.ctx.handle, C.byref(cfg), comm.handle if comm else None,
             C.byref(h))
        self.handle = h
        if comm is not None:
            comm._users.append(weakref.ref(self))

    def close(self) -> None:
        if getattr(self, "handle", None):
            call("yl_trainer_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_config(self, **kw) -> None:
        for k, v in kw.items():
            setattr(self.cfg, k, v)
        call("yl_trainer_set_config", self.handle, C.byref(self.cfg))

    # -- stepping --
    def step_device(self, frames_ptr: int, t_ptr: int, losses_ptr: int | None = None) -> None:
        call("yl_trainer_step", self.handle, C.c_void_p(frames_ptr), C.c_void_p(t_ptr),
             C.c_void_p(losses_ptr) if losses_ptr else None)

    def step_host(self, frames: np.ndarray, t: np.ndarray) -> np.ndarray:
        """frames: [3][batch][3][H][W] fp32 (ideally pinned), t: [batch] -> losses [2]."""
        fr = np.ascontiguousarray(frames, dtype=np.float32)
        tt = np.ascontiguousarray(t, dtype=np.float32)
        out = np.zeros(2, np.float32)
        call("yl_trainer_step_host", self.handle, fr.ctypes.data_as(C.c_void_p),
             tt.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p))
        return out

    def step_host_ptr(self, frames_ptr: int, t_ptr: int, out: np.ndarray) -> None:
        call("yl_trainer_step_host", self.handle, C.c_void_p(frames_ptr), C.c_void_p(t_ptr),
             out.ctypes.data_as(C.c_void_p))

    @property
    def step(self) -> int:
        """Adam step counter (steps taken so far)."""
        v = C.c_int64()
        call("yl_trainer_get_step", self.handle, C.byref(v))
        return v.value

    @step.setter
    def step(self, value: int) -> None:
        call("yl_trainer_set_step", self.handle, int(value))

    # -- parameters --
    def param_count(self, which: int) -> int:
        n = C.c_size_t()
        call("yl_trainer_param_count", self.handle, which, C.byref(n))
        return n.value

    def buffer_ptr(self, which: int, kind: int) -> int:
        p = C.c_void_p()
        call("yl_trainer_buffer", self.handle, which, kind, C.byref(p))
        return p.value

    def param_table(self, which: int) -> list[ParamEntry]:
        out, i = [], 0
        name = C.create_string_buffer(256)
        off = C.c_size_t()
        shape = (C.c_int * 4)()
        while self.L.yl_trainer_param_entry(self.handle, which, i, name, 256, C.byref(off),
                                            shape) == 0:
            out.append(ParamEntry(name.value.decode(), off.value, tuple(shape)))
            i += 1
        return out

    def download(self, which: int, kind: int = 0) -> np.ndarray:
        n = self.param_count(which)
        out = np.empty(n, np.float32)
        _memcpy_d2h(self.ctx, out, self.buffer_ptr(which, kind))
        return out

    def upload(self, which: int, data: np.ndarray, kind: int = 0) -> None:
        arr = np.ascontiguousarray(data, dtype=np.float32)
        if arr.size != self.param_count(which):
            raise YumeError(1, "parameter buffer size mismatch")
        _memcpy_h2d(self.ctx, self.buffer_ptr(which, kind), arr)
        call("yl_trainer_prepare_weights", self.handle)

    def interpolate(self, frame_a: np.ndarray, frame_b: np.ndarray, times, mode: int = 0):
        """Frames at `times` between A and B ([3][H][W] each, the trainer's size):
        mode 0 decodes the motion net's prediction, mode 1 the smoothstep lerp
        of the two encoder means.  Returns [len(times)][3][H][W]."""
        from .session import GPUTensor
        t = np.ascontiguousarray(np.asarray(times, np.float32).reshape(-1))
        fa, fb = (np.ascontiguousarray(f, dtype=np.float32).reshape(-1) for f in (frame_a, frame_b))
        h, w = self.cfg.height, self.cfg.width
        da, db = GPUTensor(self.ctx, 1, fa.size, fa), GPUTensor(self.ctx, 1, fb.size, fb)
        out = GPUTensor(self.ctx, 1, t.size * fa.size)
        call("yl_trainer_interpolate", self.handle, C.c_void_p(da.ptr), C.c_void_p(db.ptr),
             t.ctypes.data_as(C.c_void_p), t.size, int(mode), C.c_void_p(out.ptr))
        return out.toArray()[: t.size * fa.size].reshape(t.size, 3, h, w)

    def kernel_stats(self, reset: bool = False) -> dict:
        st = KernelStats()
        call("yl_trainer_kernel_stats", self.handle, C.byref(st), int(reset))
        return {CLASS_NAMES[i]: {"ms": st.ms[i], "flops": st.flops[i], "bytes": st.bytes[i],
                                 "launches": st.launches[i], "exec_flops": st.exec_flops[i]}
                for i in range(len(CLASS_NAMES))}

    def comm_stats(self, reset: bool = False) -> tuple[float, int]:
        """(exposed communication ms summed over profiled steps, steps)."""
        ms, n = C.c_double(), C.c_int()
        call("yl_trainer_comm_stats", self.handle, C.byref(ms), C.byref(n), int(reset))
        return ms.value, n.value

    def template_stats(self) -> dict:
        """Profiled conv brackets per kernel template, as of the last kernel_stats
        call: ms, algorithmic flops, executed flops, launches."""
        n = C.c_int()
        call("yl_trainer_template_stats", self.handle, None, 0, C.byref(n))
        arr = (TemplateStats * max(n.value, 1))()
        call("yl_trainer_template_stats", self.handle, arr, n.value, C.byref(n))
        return {arr[i].name.decode(): {"ms": arr[i].ms, "flops": arr[i].flops,
                                       "exec_flops": arr[i].exec_flops,
                                       "launches": arr[i].launches} for i in range(n.value)}

    def activation_bytes(self) -> int:
        b = C.c_size_t()
        call("yl_trainer_activation_bytes", self.handle, C.byref(b))
        return b.value


def interpolation_plan(seconds: float, fps: int) -> np.ndarray:
    """Frame times 0..1 of an interpolation of `seconds` at `fps`
    (interpolationFrameCount / interpolationTimes, Interpolation.swift:47-58)."""
    n = C.c_int()
    call("yl_interpolation_plan", float(seconds), int(fps), 0, None, C.byref(n))
    out = np.zeros(n.value, np.float32)
    call("yl_interpolation_plan", float(seconds), int(fps), n.value,
         out.ctypes.data_as(C.c_void_p), C.byref(n))
    return out


def _memcpy_d2h(ctx: Context, out: np.ndarray, dev_ptr: int) -> None:
    call("yl_memcpy_dtoh", ctx.handle, out.ctypes.data_as(C.c_void_p), C.c_void_p(dev_ptr),
         out.nbytes)


def _memcpy_h2d(ctx: Context, dev_ptr: int, arr: np.ndarray) -> None:
    call("yl_memcpy_htod", ctx.handle, C.c_void_p(dev_ptr), arr.ctypes.data_as(C.c_void_p),
         arr.nbytes)
