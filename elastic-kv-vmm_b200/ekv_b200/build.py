"""Build libekv_b200.so in-tree with nvcc for sm_100a.

The library is the compiled half of the package: every kernel of the data
path plus the VMM backing.  It is linked against the static CUDA runtime and
resolves driver entry points at run time, so it loads on a machine without a
GPU driver (the CPU test suite checks its exports) and needs no JIT cache.

Usage: ``python -m ekv_b200.build [--verbose] [--force] [--ptxas-info]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
REPO = PACKAGE.parents[1]
INCLUDE = REPO / "include"
BUILD_DIR = PACKAGE / "_build"
LIBRARY = PACKAGE / "lib" / "libekv_b200.so"

SOURCES = ("common.cu", "lookup.cu", "gather.cu", "migrate.cu", "swap.cu", "bitmap.cu", "shared_prefix.cu", "shadow.cu", "vmm.cpp")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")
FLAGS = ("-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-Werror=all-warnings")


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libekv_b200.so")
    return found


def _headers():
    return [*CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def _stale(target: Path, inputs) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(path.stat().st_mtime > stamp for path in inputs)


def _compile(source: Path, obj: Path, ptxas_info: bool, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(source), "-o", str(obj)]
    if ptxas_info and source.suffix == ".cu":
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{done.stdout}{done.stderr}")
    return done.stderr


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every source that changed and relink the library; return its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    jobs = []
    objects = []
    for name in SOURCES:
        source = CSRC / name
        obj = BUILD_DIR / (name + ".o")
        objects.append(obj)
        if force or ptxas_info or _stale(obj, [source, *headers]):
            jobs.append((source, obj))
    reports = []
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 1)
        with ThreadPoolExecutor(max_workers=workers) as pool:
            reports = list(pool.map(lambda job: _compile(*job, ptxas_info, verbose), jobs))
    if jobs or force or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        done = subprocess.run(cmd, capture_output=True, text=True)
        if done.returncode:
            raise RuntimeError(f"link failed:\n{done.stdout}{done.stderr}")
        os.replace(tmp, LIBRARY)
    if ptxas_info:
        for report in reports:
            sys.stdout.write(report)
    return LIBRARY


TORCH_BINDING = PACKAGE / "lib" / "_ekv_torch.so"


def build_torch_binding(verbose: bool = False, force: bool = False) -> Path | None:
    """Compile the optional pybind11 binding of the per-call lookups (csrc/torch_binding.cpp)
    against this interpreter's torch; return its path, or None (with a warning) when it
    cannot be built -- the ctypes binding then serves every call."""
    source = CSRC / "torch_binding.cpp"
    if not force and not _stale(TORCH_BINDING, [source, *INCLUDE.glob("*.h")]):
        return TORCH_BINDING
    try:
        from torch.utils.cpp_extension import load

        out = BUILD_DIR / "torch_binding"
        out.mkdir(parents=True, exist_ok=True)
        load(name="_ekv_torch", sources=[str(source)], extra_include_paths=[str(INCLUDE)],
             build_directory=str(out), with_cuda=True, verbose=verbose)
        built = out / "_ekv_torch.so"
        shutil.copy2(built, TORCH_BINDING.with_suffix(".so.tmp"))
        os.replace(TORCH_BINDING.with_suffix(".so.tmp"), TORCH_BINDING)
        return TORCH_BINDING
    except Exception as exc:  # the binding is an accelerator of the host glue, not a compute path
        print(f"warning: torch binding not built ({type(exc).__name__}: {exc})", file=sys.stderr)
        return None


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = parser.parse_args(argv)
    path = build(verbose=args.verbose, force=args.force, ptxas_info=args.ptxas_info)
    build_torch_binding(verbose=args.verbose, force=args.force)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
