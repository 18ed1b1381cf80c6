"""Build the in-tree native libraries.

    python listenflow-fastest-whisper_b200/build.py            # product library
    python listenflow-fastest-whisper_b200/build.py --oracle   # + CPU oracle (test infrastructure)

The product library ``liblffw_b200.so`` is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) next to this file, so it travels
with the source tree.  Its ``tensoracle_bundle_sha256`` symbol is the SHA-256 of
the kernel sources it was built from.
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
INCLUDE = ROOT / "include"
LIBRARY = PACKAGE / "liblffw_b200.so"
KERNEL_SOURCES = ("kernels.cu", "ptx.cuh", "launch.h")
HOST_SOURCES = ("capi.cpp",)
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return found


def bundle_digest() -> str:
    digest = hashlib.sha256()
    for name in KERNEL_SOURCES:
        digest.update(name.encode())
        digest.update((CSRC / name).read_bytes())
    return digest.hexdigest()


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    built = target.stat().st_mtime
    return any(source.stat().st_mtime > built for source in sources)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    sources = [CSRC / name for name in KERNEL_SOURCES + HOST_SOURCES] + [INCLUDE / "lffw_fp8.h"]
    if not force and not _stale(LIBRARY, sources):
        return LIBRARY
    digest = bundle_digest()
    tmp = LIBRARY.with_suffix(".so.tmp")
    command = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden",
        f"-I{INCLUDE}", f"-I{CSRC}",
        f'-DLFFW_BUNDLE_SHA256="{digest}"',
        str(CSRC / "kernels.cu"), str(CSRC / "capi.cpp"),
        "-o", str(tmp),
    ]
    if verbose:
        command.insert(1, "-Xptxas=-v")
    subprocess.run(command, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def build_oracle(force: bool = False) -> None:
    subprocess.run(["make", "-C", str(ROOT / "oracle")] + (["-B"] if force else []), check=True)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--oracle", action="store_true", help="also build the CPU oracle")
    parser.add_argument("--verbose", action="store_true", help="pass -Xptxas -v")
    args = parser.parse_args(argv)
    print(build_library(force=args.force, verbose=args.verbose))
    if args.oracle:
        build_oracle(force=args.force)
    return 0


if __name__ == "__main__":
    sys.exit(main())
