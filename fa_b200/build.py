"""Hash-keyed, idempotent nvcc build of ``libb200fa.so`` (sm_100a).

The build identity is the SHA-256 of every source under ``fa_b200/csrc``,
the public header ``include/b200fa.h``, the nvcc version line and the flag
list; the library is rebuilt only when that identity changes.  The pattern
follows the reference's CCE project build driver
(backends/cce_fa_*/project/build.py:13-116: source/compiler identity, a
manifest of artifact hashes, no partial reuse), restated for nvcc.

Runs on a CPU-only host: nvcc cross-compiles for sm_100a without a GPU.
The library goes to ``fa_b200/_build/libb200fa.so`` (in-tree, git-ignored)
so that it travels with the source tree to the GPU host.  The checking
build ``libb200fa_debug.so`` (``build(debug=True)``) is the same sources
compiled with ``-DB200FA_DEBUG``: its kernels verify coordinates, indices
and layout before use and the roles' key-block counts at exit, and report a
violation in the device status word instead of touching memory.
"""

from __future__ import annotations

import fcntl
import hashlib
import json
import os
import shutil
import subprocess
import tempfile
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_NAME = "libb200fa.so"
LIB_PATH = BUILD_DIR / LIB_NAME
MANIFEST = BUILD_DIR / "build.json"
DEBUG_LIB_NAME = "libb200fa_debug.so"
DEBUG_LIB_PATH = BUILD_DIR / DEBUG_LIB_NAME
DEBUG_MANIFEST = BUILD_DIR / "build_debug.json"
DEBUG_FLAGS = ["-DB200FA_DEBUG"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
    "-Xptxas", "-v",
]
SOURCES = ("b200fa.cu", "b200fa_causal.cu")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _nvcc_version(nvcc: str) -> str:
    out = subprocess.run([nvcc, "--version"], check=True, capture_output=True, text=True).stdout
    return out.strip().splitlines()[-1]


def _flags(debug: bool) -> list[str]:
    return NVCC_FLAGS + (DEBUG_FLAGS if debug else [])


def _paths(debug: bool) -> tuple[Path, Path]:
    return (DEBUG_LIB_PATH, DEBUG_MANIFEST) if debug else (LIB_PATH, MANIFEST)


def source_identity(nvcc: str | None = None, debug: bool = False) -> str:
    nvcc = nvcc or nvcc_path()
    h = hashlib.sha256()
    for path in sorted(CSRC.glob("*")) + sorted(INCLUDE.glob("*.h")):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    h.update(_nvcc_version(nvcc).encode())
    h.update(" ".join(_flags(debug)).encode())
    return h.hexdigest()


def _file_hash(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def is_current(debug: bool = False) -> bool:
    """True when the built library matches the current sources."""
    lib_path, manifest_path = _paths(debug)
    if not lib_path.is_file() or not manifest_path.is_file():
        return False
    try:
        manifest = json.loads(manifest_path.read_text())
        return (manifest.get("identity") == source_identity(debug=debug)
                and manifest.get("artifact_sha256") == _file_hash(lib_path))
    except (OSError, ValueError, FileNotFoundError, subprocess.CalledProcessError):
        return False


def build(force: bool = False, verbose: bool = False, debug: bool = False) -> Path:
    """Compile ``libb200fa.so`` (``debug``: ``libb200fa_debug.so``) when the
    sources changed; return its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    lib_path, manifest_path = _paths(debug)
    flags = _flags(debug)
    with open(BUILD_DIR / ".lock", "a") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and is_current(debug):
            return lib_path
        nvcc = nvcc_path()
        identity = source_identity(nvcc, debug)
        with tempfile.TemporaryDirectory(dir=BUILD_DIR) as tmp:
            out = Path(tmp) / lib_path.name
            cmd = [nvcc, *flags, f"-I{INCLUDE}", "-o", str(out),
                   *[str(CSRC / s) for s in SOURCES]]
            res = subprocess.run(cmd, capture_output=True, text=True)
            log = BUILD_DIR / ("build_debug.log" if debug else "build.log")
            log.write_text(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
            if verbose:
                print(res.stderr)
            os.replace(out, lib_path)  # never leave a partial library behind
        manifest_path.write_text(json.dumps({
            "identity": identity,
            "artifact_sha256": _file_hash(lib_path),
            "flags": flags,
            "sources": list(SOURCES),
        }, indent=2))
        return lib_path


if __name__ == "__main__":
    print(build(force=True, verbose=True))
    print(build(force=True, verbose=True, debug=True))
