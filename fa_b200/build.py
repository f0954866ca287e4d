"""Hash-keyed, idempotent nvcc build of ``libb200fa.so`` (sm_100a).

The build identity is the SHA-256 of every source under ``fa_b200/csrc``,
the public header ``include/b200fa.h``, the nvcc version line and the flag
list; the library is rebuilt only when that identity changes.  The pattern
follows the reference's CCE project build driver
(backends/cce_fa_*/project/build.py:13-116: source/compiler identity, a
manifest of artifact hashes, no partial reuse), restated for nvcc.

Runs on a CPU-only host: nvcc cross-compiles for sm_100a without a GPU.
The library goes to ``fa_b200/_build/libb200fa.so`` (in-tree, git-ignored)
so that it travels with the source tree to the GPU host.
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

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
    "-Xptxas", "-v",
]
SOURCES = ("b200fa.cu",)


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _nvcc_version(nvcc: str) -> str:
    out = subprocess.run([nvcc, "--version"], check=True, capture_output=True, text=True).stdout
    return out.strip().splitlines()[-1]


def source_identity(nvcc: str | None = None) -> str:
    nvcc = nvcc or nvcc_path()
    h = hashlib.sha256()
    for path in sorted(CSRC.glob("*")) + sorted(INCLUDE.glob("*.h")):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    h.update(_nvcc_version(nvcc).encode())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _file_hash(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def is_current() -> bool:
    """True when the built library matches the current sources."""
    if not LIB_PATH.is_file() or not MANIFEST.is_file():
        return False
    try:
        manifest = json.loads(MANIFEST.read_text())
        return (manifest.get("identity") == source_identity()
                and manifest.get("artifact_sha256") == _file_hash(LIB_PATH))
    except (OSError, ValueError, FileNotFoundError, subprocess.CalledProcessError):
        return False


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``libb200fa.so`` when the sources changed; return its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    with open(BUILD_DIR / ".lock", "a") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and is_current():
            return LIB_PATH
        nvcc = nvcc_path()
        identity = source_identity(nvcc)
        with tempfile.TemporaryDirectory(dir=BUILD_DIR) as tmp:
            out = Path(tmp) / LIB_NAME
            cmd = [nvcc, *NVCC_FLAGS, f"-I{INCLUDE}", "-o", str(out),
                   *[str(CSRC / s) for s in SOURCES]]
            res = subprocess.run(cmd, capture_output=True, text=True)
            (BUILD_DIR / "build.log").write_text(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
            if verbose:
                print(res.stderr)
            os.replace(out, LIB_PATH)  # never leave a partial library behind
        MANIFEST.write_text(json.dumps({
            "identity": identity,
            "artifact_sha256": _file_hash(LIB_PATH),
            "flags": NVCC_FLAGS,
            "sources": list(SOURCES),
        }, indent=2))
        return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
