"""Builds the attention library in-tree: rocmkernels_b200/librocmkernels_attention.so.

Every CUDA source is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
with ``-lineinfo`` so ncu can attribute counters to source lines. Objects go to
``rocmkernels_b200/_build``. The CUDA runtime is linked statically, so the library only needs
the NVIDIA driver at run time and does not depend on which libcudart the host process loaded.

Usage: ``python -m rocmkernels_b200.build [--force] [--ptxas-verbose]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
BUILD_DIR = PACKAGE / "_build"
LIBRARY = PACKAGE / "librocmkernels_attention.so"
WAIT_TEST_LIBRARY = PACKAGE / "librocmkernels_attention_waittest.so"
SOURCES = [
    "csrc/attention_abi.cu",
    "csrc/attention_tc.cu",
    "csrc/attention_tc_backward.cu",
    "csrc/copy.cu",
    "csrc/rotary.cu",
    "csrc/device.cpp",
    "csrc/context.cpp",
]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _inputs() -> list[Path]:
    files = [PACKAGE / s for s in SOURCES]
    files += sorted((PACKAGE / "csrc").glob("*.cuh")) + sorted((PACKAGE / "csrc").glob("*.h"))
    files += sorted((REPO / "include").rglob("*.h*"))
    files.append(Path(__file__))
    return files


def _compile(nvcc: str, source: Path, obj: Path, ptxas_verbose: bool, defines: tuple[str, ...] = ()) -> str:
    cmd = [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", str(REPO / "include"), "-I", str(PACKAGE / "csrc"), *(f"-D{d}" for d in defines), "-c", str(source),
           "-o", str(obj)]
    if source.suffix == ".cu":
        cmd[1:1] = ["--expt-relaxed-constexpr"]
        if ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stderr}")
    return result.stderr


def _build(library: Path, build_dir: Path, defines: tuple[str, ...], force: bool, ptxas_verbose: bool) -> Path:
    inputs = _inputs()
    if not force and library.exists():
        newest = max(p.stat().st_mtime for p in inputs if p.exists())
        if library.stat().st_mtime >= newest:
            return library
    nvcc = nvcc_path()
    build_dir.mkdir(parents=True, exist_ok=True)
    objects = [build_dir / (Path(s).name + ".o") for s in SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        logs = list(pool.map(lambda so: _compile(nvcc, PACKAGE / so[0], so[1], ptxas_verbose, defines), zip(SOURCES, objects)))
    if ptxas_verbose:
        for log in logs:
            if log:
                sys.stderr.write(log)
    tmp = library.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    os.replace(tmp, library)
    return library


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles and links the library if any input is newer than it; returns its path."""
    return _build(LIBRARY, BUILD_DIR, (), force, ptxas_verbose)


def build_wait_test(force: bool = False) -> Path:
    """The wait-test variant (librocmkernels_attention_waittest.so): the same sources built with
    RK_WAIT_TEST, whose bounded pipeline waits give up after ~0.5 ms instead of ~1 s and whose
    flash forward can be told to withhold one key tile's loads in CTA 0. Only
    tests/test_wait_timeout_gpu.py loads it, in a child process; the product library has neither."""
    return _build(WAIT_TEST_LIBRARY, BUILD_DIR / "waittest", ("RK_WAIT_TEST",), force, False)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    parser.add_argument("--wait-test", action="store_true", help="also build the wait-test variant")
    args = parser.parse_args()
    print(build(force=args.force, ptxas_verbose=args.ptxas_verbose))
    if args.wait_test:
        print(build_wait_test(force=args.force))


if __name__ == "__main__":
    main()
