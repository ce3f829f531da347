"""Ahead-of-time build of ``muspace_b200/native/libmuspace_ops.so`` for sm_100a.

Replaces the reference's ``mcc`` build of ``libmuspace_ops.so``
(``native_build.py:27-65`` in the muSPACE tree) with one ``nvcc`` link of the
MSDA sources. The CUDA runtime is linked statically, so the library loads on a
machine without a GPU (the C-ABI export checks run there) and only needs the
driver when a kernel is launched.

    python -m muspace_b200.build [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "native" / "libmuspace_ops.so"
SOURCES = ("msda_capi.cpp", "msda_forward.cu", "msda_staged.cu", "msda_backward.cu", "msda_bucketed.cu", "msda_noalloc.cu",
           "msda_deterministic.cu", "deform_agg.cu", "flash_sca.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(
        INCLUDE.glob("*.h")
    )


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs())


def build_native(force: bool = False, verbose: bool = False, output: Path | None = None,
                 defines: tuple[str, ...] = ()) -> Path:
    """Compile the MSDA library (skipped when it is newer than every source).

    ``output`` and ``defines`` (``NAME=VALUE`` macro overrides of the tuning
    constants) build a variant elsewhere; the default builds the package's own.
    """
    target = Path(output) if output is not None else LIBRARY
    if output is None and not defines and not force and up_to_date():
        return LIBRARY
    target.parent.mkdir(parents=True, exist_ok=True)
    tmp = target.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-cudart",
        "static",
        "-Xlinker",
        "--no-undefined",
        f"-I{INCLUDE}",
        *(f"-D{d}" for d in defines),
        *(str(CSRC / s) for s in SOURCES),
        "-o",
        str(tmp),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(target)
    return target


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print the command and ptxas resource usage")
    args = parser.parse_args()
    print(build_native(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
