"""Build ``libisp_b200.so`` in-tree with nvcc for sm_100a (no GPU needed)."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
OUTPUT = PACKAGE_DIR / "libisp_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    return os.fspath(candidate) if candidate.exists() else (shutil.which("nvcc") or "nvcc")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [PACKAGE_DIR.parent / "include" / "isp_b200.h"])


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    built = OUTPUT.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source into one shared object next to this file."""
    if not force and up_to_date():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-O3", "-shared", "--expt-relaxed-constexpr",
           "-I", os.fspath(PACKAGE_DIR.parent / "include"),
           "-o", os.fspath(tmp), os.fspath(CSRC / "isp_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force=True))
