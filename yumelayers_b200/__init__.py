"""yumelayers_b200 -- B200-native compute backend for YumeLayersCore's operator layer.

The product is the CUDA library ``libyumecuda.so`` (sources in ``csrc/``,
C ABI in ``include/yume_c.h``).  This package holds its ctypes binding
(``_lib``), the mirror of the reference's ``GpuSession``/``GPUTensor`` API
(``session``), the batched-op helpers (``ops``) and the training driver
(``trainer``).
"""
from ._lib import LIB_PATH, YumeError, lib  # noqa: F401

__all__ = ["LIB_PATH", "YumeError", "lib"]
