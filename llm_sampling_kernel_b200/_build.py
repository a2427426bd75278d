"""In-tree build of the two native artefacts of the package.

* ``lib/libfs_b200.so``: every CUDA kernel plus the C ABI declared in
  ``include/fused_sampling_b200.h`` (nvcc, sm_100a only, no torch).
* ``fused_sampling*.so``: the PyTorch operator module ``fused_sampling`` (C++ / pybind11) that
  mirrors the reference extension's surface and calls the C ABI.

Both land inside the package directory so that they travel with the source tree; nothing is
installed into site-packages and nothing is cached under the home directory.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
OBJDIR = PKG / "_build" / "obj"
EXTDIR = PKG / "_build" / "torch_ext"
LIBNAME = "libfs_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def header_deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def build_cuda_lib(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ for sm_100a and link lib/libfs_b200.so."""
    OBJDIR.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    headers = header_deps()
    jobs = []
    for src in cuda_sources():
        obj = OBJDIR / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [_nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(subprocess.run, cmd, capture_output=True, text=True): src for src, cmd in jobs}
            for fut in cf.as_completed(futs):
                res = fut.result()
                if res.returncode != 0:
                    raise RuntimeError(f"nvcc failed for {futs[fut].name}:\n{res.stderr}")
                if verbose and res.stderr:
                    sys.stderr.write(res.stderr)
    objs = [OBJDIR / (s.stem + ".o") for s in cuda_sources()]
    lib = LIBDIR / LIBNAME
    if force or jobs or _stale(lib, objs):
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(lib), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of {LIBNAME} failed:\n{res.stderr}")
    return lib


def _ext_filename() -> str:
    return "fused_sampling" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so")


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """Build the `fused_sampling` torch operator module next to this file."""
    src = CSRC / "torch_binding.cpp"
    target = PKG / _ext_filename()
    lib = LIBDIR / LIBNAME
    if not force and not _stale(target, [src, lib, INCLUDE / "fused_sampling_b200.h"]):
        return target
    from torch.utils import cpp_extension

    EXTDIR.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name="fused_sampling",
        sources=[str(src)],
        extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O3", "-std=c++17"],
        extra_ldflags=[f"-L{LIBDIR}", "-lfs_b200", "-Wl,-rpath,\\$$ORIGIN/lib", "-Wl,-rpath,\\$$ORIGIN/../../lib"],
        build_directory=str(EXTDIR),
        with_cuda=True,
        verbose=verbose,
        is_python_module=True,
    )
    built = EXTDIR / "fused_sampling.so"
    if not built.exists():
        found = glob.glob(str(EXTDIR / "fused_sampling*.so"))
        if not found:
            raise RuntimeError("torch extension build produced no shared object")
        built = Path(found[0])
    shutil.copy2(built, target)
    return target


def build(force: bool = False, verbose: bool = False) -> None:
    build_cuda_lib(force=force, verbose=verbose)
    build_torch_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", LIBDIR / LIBNAME, "and", PKG / _ext_filename())
