"""Build libminikv.so in-tree for sm_100a with nvcc.

    python -m myvllm_mini_engine_b200.build [--verbose]

One translation unit (csrc/abi.cu includes the kernel files), compiled with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo``.  The CUDA runtime
is linked statically, so the library only needs the NVIDIA driver at run time.

The SHA-256 of the sources (``source_hash()``) is compiled into the library
(``minikv_source_hash``).  The library is rebuilt when the hash it carries
differs from the sources' hash, never by file times, and the loader refuses a
library whose hash differs from the sources next to it.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
OUTPUT = PACKAGE / "libminikv.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "minikv.h"])


def nvcc_path():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else (shutil.which("nvcc") or "nvcc")


MARKER = b"minikv-source-hash:"


def source_hash() -> str:
    """SHA-256 over the sources' names (relative to the package root) and contents."""
    digest = hashlib.sha256()
    for src in sources():
        digest.update(src.relative_to(ROOT).as_posix().encode() + b"\0")
        digest.update(src.read_bytes() + b"\0")
    return digest.hexdigest()


def built_hash(path: Path = OUTPUT) -> str | None:
    """The source hash compiled into a built library, read from the file without loading it."""
    if not path.is_file():
        return None
    data = path.read_bytes()
    at = data.find(MARKER)
    if at < 0:
        return None
    end = at + len(MARKER)
    return data[end:end + 64].decode("ascii", errors="replace")


def up_to_date() -> bool:
    return built_hash() == source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH, *FLAGS, f'-DMINIKV_SOURCE_HASH="{source_hash()}"', "-o", str(tmp),
           str(CSRC / "abi.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr if not verbose else ''}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


def main(argv=None):
    parser = argparse.ArgumentParser(description="build libminikv.so for sm_100a")
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
