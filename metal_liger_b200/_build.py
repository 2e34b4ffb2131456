"""Build recipe for the sm_100a CUDA library behind the C ABI.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links them
into ``metal_liger_b200/lib/libmetal_liger_b200.so`` in-tree (the built
library travels with the source tree; nothing is cached elsewhere).

Usage:  python -m metal_liger_b200._build [--force] [-j N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ_DIR = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB_NAME = "libmetal_liger_b200.so"
LIB_PATH = LIB_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _digest(src: Path, extra: list[str]) -> str:
    h = hashlib.sha256()
    h.update(src.read_bytes())
    for hdr in _headers():
        h.update(hdr.name.encode())
        h.update(hdr.read_bytes())
    h.update(" ".join(extra).encode())
    return h.hexdigest()[:16]


def _compile(src: Path, extra: list[str], verbose: bool) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    tag = _digest(src, extra)
    obj = OBJ_DIR / f"{src.stem}.{tag}.o"
    if obj.exists():
        return obj
    for stale in OBJ_DIR.glob(f"{src.stem}.*.o"):
        stale.unlink()
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c",
           str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stderr.strip() or res.stdout.strip()):
        print(res.stdout + res.stderr, flush=True)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          extra_flags: list[str] | None = None) -> Path:
    """Compile and link the library; returns the path of the shared object."""
    extra = list(extra_flags or [])
    if force and OBJ_DIR.exists():
        shutil.rmtree(OBJ_DIR)
    srcs = _sources()
    jobs = jobs or min(len(srcs), max(1, os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose), srcs))
    LIB_DIR.mkdir(exist_ok=True)
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest or \
            _link_stamp() != _link_key(objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
        (LIB_DIR / ".link_key").write_text(_link_key(objs))
    return LIB_PATH


def _link_key(objs: list[Path]) -> str:
    return ",".join(sorted(o.name for o in objs))


def _link_stamp() -> str:
    p = LIB_DIR / ".link_key"
    return p.read_text() if p.exists() else ""


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
