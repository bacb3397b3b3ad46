"""Build ``libmace_b200.so`` in-tree with nvcc for sm_100a.

``python -m mace_mlx_b200.build`` (or ``__graft_entry__.build()``) compiles
every ``csrc/*.cu`` translation unit in parallel and links the shared library
next to this file, where ``native.py`` loads it from.  Objects go to
``csrc/_build/`` and are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libmace_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-Xptxas", "-O3", f"-I{INCLUDE}"]


def _nccl_include() -> list[str]:
    """nccl.h of the NCCL that torch ships (the library it dlopens at run time)."""
    try:
        import nvidia.nccl  # noqa: F401

        d = Path(list(nvidia.nccl.__path__)[0]) / "include"
        if (d / "nccl.h").exists():
            return [f"-I{d}"]
    except Exception:  # noqa: BLE001
        pass
    return []


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmace_b200")
    return cand


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    nvcc = _nvcc()
    out_dir = CSRC / "_build"
    out_dir.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    flags = FLAGS + _nccl_include() + list(extra_flags or [])
    jobs = []
    for src in sources:
        obj = out_dir / (src.stem + ".o")
        if _stale(obj, src, headers):
            jobs.append([nvcc, *ARCH, *flags, "-c", str(src), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose or res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    objs = [str(out_dir / (s.stem + ".o")) for s in sources]
    if jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart", "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of libmace_b200.so failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-info" in sys.argv else None
    print(build(verbose=v or extra is not None, extra_flags=extra))
