"""Builds the native library `boonta_b200/libboonta_b200.so` for sm_100a.

Every `.cu` file under `boonta_b200/csrc/` is compiled with nvcc
(`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`) in parallel and linked into one
shared library with a plain C ABI (`include/boonta_b200.h`). When JAXLIB_INCLUDE names
jaxlib's FFI headers (`jax.ffi.include_dir()`), `csrc/xla_ffi.cc` (the XLA FFI handlers) is
compiled into the same library. NCCL's header comes from
the nvidia-nccl wheel; the library itself is dlopen'ed at run time only when a
communicator is created. nvcc cross-compiles, so this runs without a GPU.

    python -m boonta_b200.build            # incremental
    python -m boonta_b200.build --clean    # from scratch
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libboonta_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_include() -> list[str]:
    try:
        import nvidia.nccl  # type: ignore

        inc = Path(list(nvidia.nccl.__path__)[0]) / "include"
        if (inc / "nccl.h").exists():
            return ["-I", str(inc)]
    except Exception:
        pass
    for cand in ("/usr/include", "/usr/local/cuda/include"):
        if Path(cand, "nccl.h").exists():
            return ["-I", cand]
    raise RuntimeError("nccl.h not found")


def flags() -> list[str]:
    return [
        *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-I", str(ROOT / "include"), "-I", str(CSRC), *nccl_include(),
        "-DBT_BUILD",
    ]


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), "-c", str(src), "-o", str(obj), *flags(), *extra]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(clean: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    extra = extra or []
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    # the XLA FFI handlers, only against jaxlib's own FFI headers (jax.ffi.include_dir())
    jaxlib_inc = os.environ.get("JAXLIB_INCLUDE")
    if jaxlib_inc and (Path(jaxlib_inc) / "xla" / "ffi" / "api" / "ffi.h").exists():
        sources.append(CSRC / "xla_ffi.cc")
        extra = [*extra, "-I", jaxlib_inc]
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    jobs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        for src in sources:
            obj = BUILD / (src.stem + ".o")
            if (not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
                    or extra):
                jobs.append(pool.submit(_compile, src, obj, extra))
        for job in jobs:
            obj, log = job.result()
            if verbose and log:
                print(log, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if jobs or not LIB.exists():
        cmd = [nvcc(), "-shared", *ARCH, "-o", str(LIB), *map(str, objs), "-ldl"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    lib = build(clean=args.clean or args.ptxas_info, verbose=args.verbose or args.ptxas_info,
                extra=extra)
    print(lib)


if __name__ == "__main__":
    main()
