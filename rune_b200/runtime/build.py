"""Build recipe for the engine's shared library (sm_100a).

``python -m rune_b200.runtime.build`` compiles every ``rune_b200/csrc/*.cu`` with nvcc into
``rune_b200/_lib/librune_b200.so`` (in-tree, so it travels with the source tree).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "librune_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _includes(path: Path, seen=None) -> set[Path]:
    """Local headers a source includes, directly or through other local headers."""
    import re

    seen = set() if seen is None else seen
    for name in re.findall(r'#include\s+"([^"]+)"', path.read_text()):
        dep = (path.parent / name).resolve()
        if dep.exists() and dep not in seen:
            seen.add(dep)
            _includes(dep, seen)
    return seen


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    stamp = obj.stat().st_mtime
    return any(p.stat().st_mtime > stamp for p in [src, *_includes(src)])


def needs_build() -> bool:
    if not LIB.exists():
        return True
    stamp = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "rune_b200.h"]
    return any(p.stat().st_mtime > stamp for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    build_dir = LIB_DIR / "obj"
    build_dir.mkdir(exist_ok=True)
    common = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", str(PKG.parent / "include")]
    procs = []
    for src in sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        if not force and not _stale(src, obj):
            continue  # object newer than its source and every header it includes
        cmd = common + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{out.decode()}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp)] + [str(o) for o in objs]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {res.stdout}{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
