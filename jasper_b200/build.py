"""Build recipe for libjasper_b200.so (sm_100a) and the tvm_ffi module.

Compiles every CUDA source under ``jasper_b200/csrc`` with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` into ``jasper_b200/lib``.  Objects
are rebuilt only when a source or header is newer.  Usage::

    python -m jasper_b200.build        # or jasper_b200.build.build()
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = PKG / "lib" / "obj"
ROOT = PKG.parent
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CORE_SOURCES = ["search.cu", "construct.cu", "graph.cu", "merge.cu", "capi.cu", "noalloc.cu", "dirsearch.cu", "rotate.cu", "rotate_tc.cu", "builders.cu", "rabitq.cu"]
COMMON_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I" + str(ROOT / "include")]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [NVCC, *ARCH, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")


def build(verbose: bool = False) -> Path:
    """Compile the core library; returns the path of libjasper_b200.so."""
    OBJ.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for name in CORE_SOURCES:
        src = CSRC / name
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        futs = [ex.submit(_compile, s, o, []) for s, o in jobs]
        for f in futs:
            f.result()
    so = LIB / "libjasper_b200.so"
    if jobs or not so.exists():
        cmd = [NVCC, *ARCH, "-shared", "-o", str(so), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
        if verbose:
            print("built", so)
    _build_tvm_module(so, verbose)
    return so


def _tvm_include() -> Path | None:
    try:
        import tvm_ffi
    except ImportError:
        return None
    inc = Path(tvm_ffi.__file__).resolve().parent / "include"
    return inc if inc.exists() else None


def _build_tvm_module(core: Path, verbose: bool) -> Path | None:
    """lib/libjasper_ffi.so: the reference's tvm_ffi op names over the C ABI."""
    inc = _tvm_include()
    if inc is None:
        return None
    tvm_lib = inc.parent / "lib"
    src = CSRC / "ffi_tvm.cc"
    out = LIB / "libjasper_ffi.so"
    if out.exists() and out.stat().st_mtime > max(src.stat().st_mtime, core.stat().st_mtime,
                                                    _headers_mtime()):
        return out
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-o", str(out), str(src),
           f"-I{inc}", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
           f"-L{LIB}", "-ljasper_b200", f"-L{tvm_lib}", "-ltvm_ffi",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tvm_lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("tvm_ffi module build failed:\n" + r.stderr)
    if verbose:
        print("built", out)
    return out


if __name__ == "__main__":
    print(build(verbose=True))
    sys.exit(0)
