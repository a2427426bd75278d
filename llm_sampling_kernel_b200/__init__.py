"""B200-native (sm_100a) fused top-k / top-p token sampler.

Hot path: ``[B, V]`` FP16/BF16 logits -> ``[B]`` int64 token ids in one kernel launch.

Layers, bottom up:

* ``lib/libfs_b200.so`` -- the CUDA kernels and the C ABI (``include/fused_sampling_b200.h``).
* ``fused_sampling`` -- the PyTorch operator module with the reference extension's surface
  (``sample_fused``, ``topk_fused``, ``stages_fused``, ``probe_phase``, ``kernel_attrs``,
  ``probe_noop``, ``probe_scan_rowblock``, ``probe_scan_split``) plus extensions.
* :mod:`llm_sampling_kernel_b200.fused` -- the Python front end (same signatures as the
  reference's ``benchmarks/fused.py``).
* :mod:`llm_sampling_kernel_b200.abi` -- a ctypes binding of the C ABI.
* :mod:`llm_sampling_kernel_b200.sharded` -- batch-sharded and vocab-sharded multi-GPU use.

There is no CPU fallback: if the native modules are missing, importing the operator module
raises.
"""

from __future__ import annotations

import ctypes
import importlib
from pathlib import Path

__version__ = "1.0.0"

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libfs_b200.so"

_lib_handle = None
_ops = None


def native_library() -> ctypes.CDLL:
    """The loaded C-ABI library (``lib/libfs_b200.so``); raises if it was not built."""
    global _lib_handle
    if _lib_handle is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m llm_sampling_kernel_b200._build`"
            )
        _lib_handle = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    return _lib_handle


def ops():
    """The ``fused_sampling`` operator module (torch extension); raises if it was not built."""
    global _ops
    if _ops is None:
        import torch  # noqa: F401  (loads libc10 / libtorch for the extension)

        native_library()
        try:
            _ops = importlib.import_module("llm_sampling_kernel_b200.fused_sampling")
        except ImportError as e:
            raise ImportError(
                "the fused_sampling extension is not built: run `python -m llm_sampling_kernel_b200._build`"
            ) from e
    return _ops
