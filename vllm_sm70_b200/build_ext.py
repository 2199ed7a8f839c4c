"""Native build driver for ``vllm_sm70_b200/_b200_C.so``.

The extension is compiled for exactly one target, ``sm_100a`` (B200): every
``.cu`` under ``csrc/`` gets ``-gencode arch=compute_100a,code=sm_100a`` and
nothing else, so torch's own arch list never leaks in. Host-only ``.cpp``
files are compiled by g++ against the torch headers. The build is driven by
a generated ``build.ninja`` in ``_build/`` (incremental, parallel); the
product is an in-tree ``.so`` that ``_ext.load()`` opens with
``torch.ops.load_library``.

Reference parity: ``sm70/setup.py:54-81`` + ``sm70/CMakeLists.txt:151-155``
(one extension, one arch, offline build). Differences: the reference pins
``code=sm_70`` through CMake; this driver pins ``code=sm_100a`` through ninja.

Usage::

    python -m vllm_sm70_b200.build_ext            # build (incremental)
    python -m vllm_sm70_b200.build_ext --clean    # rebuild from scratch
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = REPO_DIR / "_build"
SO_PATH = PKG_DIR / "_b200_C.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and Path(cand, "bin", "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _torch_paths() -> tuple[list[str], list[str], bool]:
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths(device_type="cuda")
    lib = cpp_extension.library_paths(device_type="cuda")
    return inc, lib, bool(torch._C._GLIBCXX_USE_CXX11_ABI)


def _sources() -> tuple[list[Path], list[Path]]:
    cu = sorted(CSRC.rglob("*.cu"))
    cpp = sorted(CSRC.rglob("*.cpp"))
    return cu, cpp


def write_ninja(debug_bounds: bool = False) -> Path:
    cuda = _cuda_home()
    inc, lib, abi = _torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    cu, cpp = _sources()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={int(abi)}", "-DTORCH_EXTENSION_NAME=_b200_C",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
    if debug_bounds:
        defs.append("-DB200_DEBUG_BOUNDS=1")
    incs = [f"-I{CSRC}"] + [f"-I{p}" for p in inc] + [f"-I{py_inc}", f"-I{cuda}/include"]
    nvcc_flags = ARCH_FLAGS + [
        "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-Wno-deprecated-declarations",
        "-DNDEBUG", "--threads", "2",
        # -Xptxas -v prints registers/spills/smem per kernel into _build/*.log
        "-Xptxas", "-v",
    ] + defs + incs
    cxx_flags = ["-O3", "-std=c++17", "-fPIC", "-DNDEBUG", "-Wno-deprecated-declarations",
                 "-Wno-unused-function"] + defs + incs
    ldflags = ["-shared"] + [f"-L{p}" for p in lib] + [f"-L{cuda}/lib64"] + [
        "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lcudart",
    ] + [f"-Wl,-rpath,{p}" for p in lib]

    def q(xs):
        return " ".join(xs)

    lines = [
        "ninja_required_version = 1.3",
        f"nvcc = {cuda}/bin/nvcc",
        "cxx = g++",
        f"nvcc_flags = {q(nvcc_flags)}",
        f"cxx_flags = {q(cxx_flags)}",
        f"ldflags = {q(ldflags)}",
        "rule nvcc",
        "  command = $nvcc $nvcc_flags -MD -MF $out.d -c $in -o $out > $out.log 2>&1 || (cat $out.log; exit 1)",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $in",
        "rule cxx",
        "  command = $cxx $cxx_flags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule link",
        "  command = $cxx $in $ldflags -o $out",
        "  description = LINK $out",
    ]
    objs = []
    for src in cu + cpp:
        rel = src.relative_to(CSRC)
        obj = BUILD_DIR / (str(rel).replace("/", "__") + ".o")
        objs.append(obj)
        rule = "nvcc" if src.suffix == ".cu" else "cxx"
        lines.append(f"build {obj}: {rule} {src}")
    lines.append(f"build {SO_PATH}: link {' '.join(map(str, objs))}")
    lines.append(f"default {SO_PATH}")
    path = BUILD_DIR / "build.ninja"
    text = "\n".join(lines) + "\n"
    if not path.exists() or path.read_text() != text:
        path.write_text(text)
    return path


def build(clean: bool = False, jobs: int | None = None, debug_bounds: bool = False,
          verbose: bool = False) -> Path:
    if clean and BUILD_DIR.exists():
        shutil.rmtree(BUILD_DIR)
    ninja_file = write_ninja(debug_bounds=debug_bounds)
    jobs = jobs or max(1, min(os.cpu_count() or 1, 16))
    cmd = ["ninja", "-f", str(ninja_file), "-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    res = subprocess.run(cmd, cwd=BUILD_DIR, capture_output=not verbose, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError(f"_b200_C build failed:\n{out[-20000:]}")
    return SO_PATH


def ptxas_report() -> str:
    """Concatenate the ``-Xptxas -v`` logs (registers, spills, smem per kernel)."""
    logs = sorted(BUILD_DIR.glob("*.o.log"))
    return "\n".join(p.read_text() for p in logs)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--debug-bounds", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v summary")
    args = ap.parse_args(argv)
    so = build(clean=args.clean, jobs=args.jobs, debug_bounds=args.debug_bounds,
               verbose=args.verbose)
    print(f"built {so}")
    if args.ptxas:
        print(ptxas_report())
    return 0


if __name__ == "__main__":
    sys.exit(main())
