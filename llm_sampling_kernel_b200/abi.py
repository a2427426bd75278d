"""ctypes binding of the C ABI in ``include/fused_sampling_b200.h``.

This is the binding a caller without the torch extension uses (and what the parity tests call
through): plain pointers and sizes. The helpers here accept torch CUDA tensors for convenience
and pass only their device pointers, the current stream and sizes across the boundary.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import native_library

FS_OK, FS_EINVAL, FS_EUNSUPPORTED, FS_ELAUNCH, FS_ETIMEOUT, FS_EWORKSPACE = range(6)
FS_F16, FS_BF16 = 0, 1
FS_NUM_PHASES = 7
STATUS_NAMES = {
    FS_OK: "FS_OK",
    FS_EINVAL: "FS_EINVAL",
    FS_EUNSUPPORTED: "FS_EUNSUPPORTED",
    FS_ELAUNCH: "FS_ELAUNCH",
    FS_ETIMEOUT: "FS_ETIMEOUT",
    FS_EWORKSPACE: "FS_EWORKSPACE",
}

# Every entry point declared in include/fused_sampling_b200.h.
EXPORTED = (
    "fs_sample",
    "fs_topk",
    "fs_probe_phase",
    "fs_shard_candidates",
    "fs_merge_sample",
    "fs_probe_noop",
    "fs_probe_scan_rowblock",
    "fs_probe_scan_split",
    "fs_kernel_attrs",
    "fs_last_error",
    "fs_plan",
    "fs_version",
    "fs_workspace_size",
    "fs_sample_noalloc",
    "fs_tp_merge_sample",
    "fs_ipc_alloc",
    "fs_ipc_free",
    "fs_ipc_handle",
    "fs_ipc_open",
    "fs_ipc_close",
)
FS_IPC_HANDLE_BYTES = 64
FS_PATH_AUTO, FS_PATH_CLUSTER, FS_PATH_STREAM, FS_PATH_WIDE = 0, 1, 2, 3
FS_INPUT_READY = 1  # fs_sample_args.input_flags: the logits are complete when the call is enqueued


class FsRng(ctypes.Structure):
    _fields_ = [
        ("uniforms", ctypes.c_void_p),
        ("seed", ctypes.c_uint64),
        ("offset", ctypes.c_uint64),
        ("seed_ptr", ctypes.c_void_p),
        ("offset_ptr", ctypes.c_void_p),
        ("offset_intragraph", ctypes.c_uint64),
        ("row_base", ctypes.c_int64),
    ]


class FsSampleArgs(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("vocab", ctypes.c_int64),
        ("row_stride", ctypes.c_int64),
        ("id_base", ctypes.c_int64),
        ("top_k", ctypes.c_int64),
        ("top_p", ctypes.c_float),
        ("top_k_rows", ctypes.c_void_p),
        ("top_p_rows", ctypes.c_void_p),
        ("rng", FsRng),
        ("out_ids", ctypes.c_void_p),
        ("topk_ids", ctypes.c_void_p),
        ("keep", ctypes.c_void_p),
        ("renormed", ctypes.c_void_p),
        ("row_status", ctypes.c_void_p),
        ("splits", ctypes.c_int32),
        ("stop_phase", ctypes.c_int32),
        ("path", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64),
        ("temperature", ctypes.c_float),
        ("input_flags", ctypes.c_uint32),
    ]


class FsTpPeers(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("max_batch", ctypes.c_int64),
        ("epoch", ctypes.c_uint32),
        ("wait_polls", ctypes.c_int64),
        ("recv", ctypes.c_void_p),
        ("flags", ctypes.c_void_p),
        ("peer_recv", ctypes.c_void_p),
        ("peer_flags", ctypes.c_void_p),
        ("epoch_counter", ctypes.c_void_p),
    ]


class FsKernelAttr(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 64),
        ("param", ctypes.c_int32),
        ("block", ctypes.c_int32),
        ("regs", ctypes.c_int32),
        ("local_bytes", ctypes.c_int32),
        ("static_smem", ctypes.c_int32),
        ("blocks_per_sm", ctypes.c_int32),
    ]


class FsPlanInfo(ctypes.Structure):
    _fields_ = [
        ("splits", ctypes.c_int32),
        ("chunks", ctypes.c_int32),
        ("threads", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("maxima_per_thread", ctypes.c_int32),
        ("lanes_per_max", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("path", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_uint64),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = native_library()
        P = ctypes.POINTER
        L.fs_sample.argtypes = [P(FsSampleArgs), ctypes.c_void_p]
        L.fs_topk.argtypes = [P(FsSampleArgs), ctypes.c_void_p]
        L.fs_probe_phase.argtypes = [P(FsSampleArgs), ctypes.c_void_p]
        L.fs_shard_candidates.argtypes = [P(FsSampleArgs), ctypes.c_void_p, ctypes.c_void_p]
        L.fs_merge_sample.argtypes = [P(FsSampleArgs), ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        L.fs_probe_noop.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.fs_probe_scan_rowblock.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        L.fs_probe_scan_split.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
        L.fs_kernel_attrs.argtypes = [P(FsKernelAttr), ctypes.c_int32]
        L.fs_kernel_attrs.restype = ctypes.c_int32
        L.fs_last_error.restype = ctypes.c_char_p
        L.fs_version.restype = ctypes.c_char_p
        L.fs_plan.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, P(FsPlanInfo)]
        L.fs_workspace_size.argtypes = [P(FsSampleArgs)]
        L.fs_workspace_size.restype = ctypes.c_uint64
        L.fs_sample_noalloc.argtypes = [P(FsSampleArgs), ctypes.c_void_p]
        L.fs_tp_merge_sample.argtypes = [P(FsSampleArgs), ctypes.c_void_p, P(FsTpPeers), ctypes.c_void_p]
        L.fs_ipc_alloc.argtypes = [ctypes.c_uint64, P(ctypes.c_void_p)]
        L.fs_ipc_free.argtypes = [ctypes.c_void_p]
        L.fs_ipc_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.fs_ipc_open.argtypes = [ctypes.c_void_p, P(ctypes.c_void_p)]
        L.fs_ipc_close.argtypes = [ctypes.c_void_p]
        for name in ("fs_tp_merge_sample", "fs_ipc_alloc", "fs_ipc_free", "fs_ipc_handle", "fs_ipc_open", "fs_ipc_close",
                     "fs_sample", "fs_sample_noalloc", "fs_topk", "fs_probe_phase", "fs_shard_candidates", "fs_merge_sample",
                     "fs_probe_noop", "fs_probe_scan_rowblock", "fs_probe_scan_split", "fs_plan"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


class FsError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = lib().fs_last_error().decode(errors="replace")
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}: {msg}")


def check(status: int, what: str) -> None:
    if status != FS_OK:
        raise FsError(status, what)


def version() -> str:
    return lib().fs_version().decode()


@dataclass
class Plan:
    splits: int
    chunks: int
    threads: int
    capacity: int
    maxima_per_thread: int
    lanes_per_max: int
    smem_bytes: int
    path: int
    workspace_bytes: int


def plan(batch: int, vocab: int, top_k: int, splits: int = 0) -> Plan:
    info = FsPlanInfo()
    check(lib().fs_plan(batch, vocab, top_k, splits, ctypes.byref(info)), "fs_plan")
    return Plan(info.splits, info.chunks, info.threads, info.capacity, info.maxima_per_thread,
                info.lanes_per_max, info.smem_bytes, info.path, info.workspace_bytes)


def kernel_attrs() -> list[tuple]:
    n = lib().fs_kernel_attrs(None, 0)
    rows = (FsKernelAttr * n)()
    lib().fs_kernel_attrs(rows, n)
    return [(r.name.decode(), r.param, r.block, r.regs, r.local_bytes, r.static_smem, r.blocks_per_sm)
            for r in rows]


# ---- tensor convenience (device pointers only cross the boundary) ---------------------------


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def make_args(logits, top_k: int, top_p: float = 1.0, *, seed: int = 0, offset: int = 0, uniforms=None,
              top_k_rows=None, top_p_rows=None, id_base: int = 0, row_base: int = 0, splits: int = 0,
              out_ids=None, topk_ids=None, keep=None, renormed=None, row_status=None,
              stop_phase: int = 0, path: int = FS_PATH_AUTO, temperature: float = 1.0) -> FsSampleArgs:
    import torch

    a = FsSampleArgs()
    if logits is not None:
        if logits.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError("logits must be float16 or bfloat16")
        a.logits = logits.data_ptr()
        a.dtype = FS_BF16 if logits.dtype == torch.bfloat16 else FS_F16
        a.batch = logits.shape[0]
        a.vocab = logits.shape[1]
        a.row_stride = logits.stride(0)
    a.id_base = id_base
    a.top_k = top_k
    a.top_p = top_p
    a.top_k_rows = None if top_k_rows is None else top_k_rows.data_ptr()
    a.top_p_rows = None if top_p_rows is None else top_p_rows.data_ptr()
    a.rng.uniforms = None if uniforms is None else uniforms.data_ptr()
    a.rng.seed = seed & ((1 << 64) - 1)
    a.rng.offset = offset & ((1 << 64) - 1)
    a.rng.row_base = row_base
    a.out_ids = None if out_ids is None else out_ids.data_ptr()
    a.topk_ids = None if topk_ids is None else topk_ids.data_ptr()
    a.keep = None if keep is None else keep.data_ptr()
    a.renormed = None if renormed is None else renormed.data_ptr()
    a.row_status = None if row_status is None else row_status.data_ptr()
    a.splits = splits
    a.stop_phase = stop_phase
    a.path = path
    a.temperature = temperature
    return a


def attach_workspace(a: FsSampleArgs, device):
    """Allocates the workspace the call needs (None when it needs none) and records it in `a`.
    Keep the returned tensor alive until the call's work has run (stream order)."""
    import torch

    n = lib().fs_workspace_size(ctypes.byref(a))
    if n == 0:
        return None
    ws = torch.empty(n, dtype=torch.uint8, device=device)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = n
    return ws


def sample(logits, top_k: int, top_p: float, *, seed: int = 0, offset: int = 0, uniforms=None,
           top_k_rows=None, top_p_rows=None, splits: int = 0, id_base: int = 0, row_base: int = 0,
           stages: bool = False, path: int = FS_PATH_AUTO, stream=None, temperature: float = 1.0):
    """fs_sample through ctypes. Returns ids, or (ids, topk_ids, keep, renormed, status)."""
    import torch

    B, V = logits.shape
    K = min(top_k, V)
    dev = logits.device
    out = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    ids = keep = ren = None
    if stages:
        ids = torch.empty(B, K, dtype=torch.int64, device=dev)
        keep = torch.empty(B, K, dtype=torch.uint8, device=dev)
        ren = torch.empty(B, K, dtype=torch.float32, device=dev)
    a = make_args(logits, top_k, top_p, seed=seed, offset=offset, uniforms=uniforms, top_k_rows=top_k_rows,
                  top_p_rows=top_p_rows, id_base=id_base, row_base=row_base, splits=splits, out_ids=out,
                  topk_ids=ids, keep=keep, renormed=ren, row_status=status, path=path, temperature=temperature)
    ws = attach_workspace(a, dev)  # noqa: F841  (alive until the launches are enqueued)
    check(lib().fs_sample(ctypes.byref(a), _stream(stream)), "fs_sample")
    if stages:
        return out, ids, keep.bool(), ren, status
    return out


def topk(logits, top_k: int, *, splits: int = 0, path: int = FS_PATH_AUTO, stream=None):
    import torch

    B, V = logits.shape
    K = min(top_k, V)
    ids = torch.empty(B, K, dtype=torch.int64, device=logits.device)
    a = make_args(logits, top_k, 1.0, splits=splits, topk_ids=ids, path=path)
    ws = attach_workspace(a, logits.device)  # noqa: F841
    check(lib().fs_topk(ctypes.byref(a), _stream(stream)), "fs_topk")
    return ids


def shard_candidates(logits, top_k: int, id_base: int, *, splits: int = 0, out=None, stream=None):
    import torch

    B = logits.shape[0]
    cand = out if out is not None else torch.empty(B, top_k + 1, dtype=torch.int64, device=logits.device)
    a = make_args(logits, top_k, 1.0, id_base=id_base, splits=splits)
    ws = attach_workspace(a, logits.device)  # noqa: F841
    check(lib().fs_shard_candidates(ctypes.byref(a), _ptr(cand), _stream(stream)), "fs_shard_candidates")
    return cand


def merge_sample(cand, bf16: bool, top_k: int, top_p: float, *, seed: int = 0, offset: int = 0, uniforms=None,
                 row_base: int = 0, stream=None):
    """cand: int64 [parts, B, top_k + 1]. Returns (ids, status)."""
    import torch

    parts, B, _ = cand.shape
    out = torch.empty(B, dtype=torch.int64, device=cand.device)
    status = torch.empty(B, dtype=torch.int32, device=cand.device)
    a = make_args(None, top_k, top_p, seed=seed, offset=offset, uniforms=uniforms, row_base=row_base,
                  out_ids=out, row_status=status)
    a.dtype = FS_BF16 if bf16 else FS_F16
    a.batch = B
    check(lib().fs_merge_sample(ctypes.byref(a), _ptr(cand), parts, _stream(stream)), "fs_merge_sample")
    return out, status


# ---- peer buffers for the tensor-parallel exchange (set-up time only) ------------------------


class _CudaBuffer:
    """A raw device allocation seen as a tensor (zero copy, __cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2}


def ipc_alloc(shape, dtype) -> tuple:
    """A zeroed device buffer of its own allocation on the current device: (tensor, pointer)."""
    import torch

    typestr = {torch.int64: "<i8", torch.int32: "<i4"}[dtype]
    n = 1
    for d in shape:
        n *= d
    ptr = ctypes.c_void_p()
    check(lib().fs_ipc_alloc(n * (8 if dtype == torch.int64 else 4), ctypes.byref(ptr)), "fs_ipc_alloc")
    t = torch.as_tensor(_CudaBuffer(ptr.value, shape, typestr), device="cuda")
    return t, ptr.value


def ipc_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(FS_IPC_HANDLE_BYTES)
    check(lib().fs_ipc_handle(ctypes.c_void_p(ptr), buf), "fs_ipc_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    check(lib().fs_ipc_open(ctypes.create_string_buffer(handle, FS_IPC_HANDLE_BYTES), ctypes.byref(ptr)),
          "fs_ipc_open")
    return ptr.value


def ipc_close(ptr: int) -> None:
    check(lib().fs_ipc_close(ctypes.c_void_p(ptr)), "fs_ipc_close")


def ipc_free(ptr: int) -> None:
    check(lib().fs_ipc_free(ctypes.c_void_p(ptr)), "fs_ipc_free")
