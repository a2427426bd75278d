"""The C-ABI library loads and exports exactly what include/fused_sampling_b200.h declares, and
its host-only entry points (plan, version, argument validation) behave. CPU only: no compute."""

import ctypes
import re
from pathlib import Path

import pytest

from llm_sampling_kernel_b200 import abi

HEADER = Path(__file__).resolve().parents[1] / "include" / "fused_sampling_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^FS_API\s+[\w\s\*]+?\b(fs_\w+)\(", text, flags=re.M)))


def test_header_declares_the_documented_entry_points():
    assert declared_functions() == sorted(abi.EXPORTED)


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_every_declared_symbol(name):
    lib = abi.lib()
    assert hasattr(lib, name), f"{name} missing from libfs_b200.so"
    assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_version_names_the_target():
    assert "sm_100a" in abi.version()


def test_struct_layout_matches_the_header(tmp_path):
    # offsets of every field as the C compiler lays them out, against the ctypes mirror
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"fs_sample_args": abi.FsSampleArgs, "fs_rng": abi.FsRng, "fs_kernel_attr": abi.FsKernelAttr,
               "fs_plan_info": abi.FsPlanInfo, "fs_tp_peers": abi.FsTpPeers}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    for line in filter(None, out):
        cname, field, value = line.split()
        cls = structs[cname]
        got = ctypes.sizeof(cls) if field == "sizeof" else getattr(cls, field).offset
        assert got == int(value), f"{cname}.{field}: ctypes {got} vs C {value}"


def test_plan_table():
    p = abi.plan(1, 151936, 50)
    assert (p.splits, p.chunks, p.threads) == (16, 5, 256)
    assert p.splits * p.chunks * p.threads * 8 >= 151936
    q = abi.plan(1024, 151936, 50)
    assert q.path == abi.FS_PATH_STREAM and q.workspace_bytes > 0
    assert q.splits * q.chunks * q.threads * 8 >= 151936
    assert q.smem_bytes <= 227 * 1024
    r = abi.plan(8, 151936, 1024)
    assert r.capacity >= 4 * 1024
    assert r.splits * r.threads * r.maxima_per_thread // r.lanes_per_max >= 4 * 1024
    small = abi.plan(16, 4001, 100)
    assert small.splits * small.chunks * small.threads * 8 >= 4001
    for B in (1, 4, 16, 64, 1024):
        for V in (2000, 4001, 32000, 128256, 151936, 256000):
            for k in (1, 50, 256, 1024):
                pl = abi.plan(B, V, k)
                assert pl.splits * pl.chunks * pl.threads * 8 >= V
                assert 1 <= pl.splits <= 16
                assert pl.capacity >= min(k, V)


def test_top_k_beyond_the_survivor_buffer_plans_the_wide_path():
    for B in (1, 8, 64, 1024):
        for V, k in ((151936, 151936), (151936, 8193), (128256, 20000), (256000, 1 << 20)):
            pl = abi.plan(B, V, k)
            assert pl.path == abi.FS_PATH_WIDE, (B, V, k)
            # a [B, 65536] per-key count histogram and a few words per row and slice
            assert B * 65536 * 4 < pl.workspace_bytes < B * 65536 * 4 + B * 1024 + 4096
            assert pl.splits * pl.chunks * pl.threads * 8 >= V
    assert abi.plan(8, 151936, 8192).path == abi.FS_PATH_CLUSTER


def test_plan_rejects_a_vocabulary_beyond_the_register_budget():
    with pytest.raises(abi.FsError) as e:
        abi.plan(1, 1 << 21, 50)
    assert e.value.status == abi.FS_EUNSUPPORTED


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype = 7
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EINVAL
    assert "float16 or bfloat16" in lib.fs_last_error().decode()
    a.dtype = abi.FS_BF16
    a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = 2, 100, 100, 5, 1.5
    a.logits = 0x1000
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EINVAL
    assert "top_p must be in (0, 1]" in lib.fs_last_error().decode()
    a.top_p, a.top_k = 0.9, 0
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EINVAL
    assert "top_k must be >= 1" in lib.fs_last_error().decode()
    a.top_k, a.row_stride = 5, 50
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EINVAL
    a.row_stride, a.stop_phase = 100, 9
    assert lib.fs_probe_phase(ctypes.byref(a), None) == abi.FS_EINVAL
    assert "phase must be in [1, 7]" in lib.fs_last_error().decode()
    assert lib.fs_sample(None, None) == abi.FS_EINVAL
    assert lib.fs_probe_noop(None, 4, None) == abi.FS_EINVAL
    assert lib.fs_merge_sample(ctypes.byref(a), None, 2, None) == abi.FS_EINVAL


def test_large_batches_plan_the_streaming_path_with_a_workspace():
    big = abi.plan(1024, 151936, 50)
    assert big.path == abi.FS_PATH_STREAM
    # [B, S, M] packed candidates (M >= 2k) + [B, S] counts + alignment slack
    assert big.workspace_bytes >= 1024 * big.splits * (2 * 50 * 8 + 4)
    assert abi.plan(1, 151936, 50).path == abi.FS_PATH_CLUSTER
    # AUTO (measured crossovers with the cluster path at its measured split): k <= 128 from 96
    # rows; 128 < k <= 256 from 64 rows when the row needs 8 or more CTAs, else from 96
    assert abi.plan(95, 151936, 50).path == abi.FS_PATH_CLUSTER
    assert abi.plan(96, 151936, 50).path == abi.FS_PATH_STREAM
    assert abi.plan(63, 151936, 200).path == abi.FS_PATH_CLUSTER
    assert abi.plan(64, 151936, 200).path == abi.FS_PATH_STREAM
    assert abi.plan(64, 128256, 200).path == abi.FS_PATH_CLUSTER
    assert abi.plan(96, 128256, 256).path == abi.FS_PATH_STREAM
    assert abi.plan(1024, 151936, 256).path == abi.FS_PATH_STREAM
    assert abi.plan(1, 151936, 50).workspace_bytes == 0
    # beyond the streaming path's k the cluster path serves every batch size
    assert abi.plan(1024, 151936, 1024).path == abi.FS_PATH_CLUSTER


def test_the_split_table_follows_the_measured_sweep():
    """CTAs per row from the B200 sweep: more CTAs only while the batch leaves SMs idle, the
    fewest that hold the row once it does (4 for V <= 131072, else 8); the streaming path always
    takes the fewest slices that hold the row."""
    assert abi.plan(1, 151936, 50).splits == 16
    assert abi.plan(16, 151936, 50).splits == 8
    assert abi.plan(32, 128256, 50).splits == 8
    assert abi.plan(32, 128256, 256).splits == 4
    assert abi.plan(64, 128256, 50).splits == 4
    assert abi.plan(64, 151936, 50).splits == 8
    assert abi.plan(16, 128256, 1024).splits == 4
    assert abi.plan(1024, 151936, 50).splits == 8     # streaming
    assert abi.plan(1024, 128256, 50).splits == 4     # streaming
    assert abi.plan(4, 2000, 50).splits == 1          # one chunk per CTA covers the row
    assert abi.plan(8, 151936, 50, 4).splits == 8     # a request the registers cannot hold is raised


def test_the_forced_streaming_path_plans_a_workspace():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype, a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = abi.FS_BF16, 1024, 151936, 151936, 50, 0.9
    a.path = abi.FS_PATH_STREAM
    # [B, S, M] packed candidates (M >= 2k) + [B, S] counts + alignment slack, S >= 8 slices
    assert lib.fs_workspace_size(ctypes.byref(a)) >= 1024 * 8 * (2 * 50 * 8 + 4)


def test_workspace_size_follows_the_plan_and_the_path_override():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype, a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = abi.FS_BF16, 1024, 151936, 151936, 50, 0.9
    assert lib.fs_workspace_size(ctypes.byref(a)) == abi.plan(1024, 151936, 50).workspace_bytes > 0
    a.path = abi.FS_PATH_CLUSTER
    assert lib.fs_workspace_size(ctypes.byref(a)) == 0
    a.path = abi.FS_PATH_WIDE
    assert lib.fs_workspace_size(ctypes.byref(a)) >= 1024 * 65536 * 4
    a.path, a.batch = abi.FS_PATH_STREAM, 1
    assert lib.fs_workspace_size(ctypes.byref(a)) > 0
    assert lib.fs_workspace_size(None) == 0


def test_the_streaming_path_without_its_workspace_is_rejected_before_any_launch():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype, a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = abi.FS_BF16, 1024, 151936, 151936, 50, 0.9
    a.logits = 0x1000
    a.out_ids = 0x2000
    a.path = abi.FS_PATH_STREAM
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EWORKSPACE
    assert "workspace" in lib.fs_last_error().decode()
    a.workspace, a.workspace_bytes = 0x3000, 64
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EWORKSPACE
    a.path, a.top_k = abi.FS_PATH_STREAM, 1024
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EUNSUPPORTED


def test_unknown_paths_and_unsupported_forced_paths_are_rejected():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype, a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = abi.FS_BF16, 4, 151936, 151936, 50, 0.9
    a.logits, a.out_ids = 0x1000, 0x2000
    a.path = 9
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EINVAL
    assert "path" in lib.fs_last_error().decode()
    # k beyond the survivor buffer: the cluster and streaming paths refuse it, AUTO goes wide
    a.path, a.top_k = abi.FS_PATH_CLUSTER, 151936
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EUNSUPPORTED
    assert "capacity" in lib.fs_last_error().decode()
    a.path = abi.FS_PATH_STREAM
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EUNSUPPORTED
    # the wide path produces token ids and row status only
    a.path, a.topk_ids = abi.FS_PATH_AUTO, 0x3000
    assert lib.fs_sample(ctypes.byref(a), None) == abi.FS_EUNSUPPORTED
    assert "wide path" in lib.fs_last_error().decode()
    a.topk_ids, a.top_k, a.path = None, 50, abi.FS_PATH_WIDE
    assert lib.fs_topk(ctypes.byref(a), None) == abi.FS_EINVAL  # (topk_ids is required)
    a.topk_ids = 0x3000
    assert lib.fs_topk(ctypes.byref(a), None) == abi.FS_EUNSUPPORTED


def test_peer_exchange_arguments_are_checked_before_any_launch():
    lib = abi.lib()
    a = abi.FsSampleArgs()
    a.dtype, a.batch, a.vocab, a.row_stride, a.top_k, a.top_p = abi.FS_BF16, 4, 128000, 128000, 64, 0.9
    a.out_ids = 0x2000
    tp = abi.FsTpPeers()
    tp.world, tp.rank, tp.max_batch, tp.epoch = 2, 0, 4, 1
    tp.recv, tp.flags, tp.peer_recv, tp.peer_flags = 0x3000, 0x4000, 0x5000, 0x6000
    assert lib.fs_tp_merge_sample(ctypes.byref(a), None, ctypes.byref(tp), None) == abi.FS_EINVAL
    cand = 0x7000
    for field, bad in (("rank", 2), ("epoch", 0), ("max_batch", 3), ("world", 0), ("recv", None)):
        saved = getattr(tp, field)
        setattr(tp, field, bad)
        assert lib.fs_tp_merge_sample(ctypes.byref(a), cand, ctypes.byref(tp), None) == abi.FS_EINVAL, field
        setattr(tp, field, saved)
    assert "epoch" in lib.fs_last_error().decode()
    assert lib.fs_ipc_handle(None, None) == abi.FS_EINVAL
    assert lib.fs_ipc_open(None, None) == abi.FS_EINVAL
    assert lib.fs_ipc_close(None) == abi.FS_EINVAL
