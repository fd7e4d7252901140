"""Builds the CPU checkers (TEST INFRASTRUCTURE, never linked into the product).

    python oracle/build.py [--reference <root>]

  oracle/liboracle.so        the C++ restatement of the 3DGS path (oracle/gs3d_oracle.cpp), OpenMP,
                             compiled with -ffp-contract=off so float32 rounding follows the source
  oracle/_ref/libsplat2d_ref.so   the reference's own splat2d CPU code (phase0/csrc/macrotile/
                             splat2d_cpu.cpp, compiled in place from the reference tree with g++)
                             behind oracle/splat2d_ref_capi.cpp; built only where the reference
                             tree exists (REFERENCE_ROOT or --reference)
  oracle/_ref/gs2d_cuda_ref/gs2d_cuda_ref.so   the reference's own toy2d CUDA rasterizer
                             (toy2d/csrc/rasterize.cu, the extension toy2d/gs2d/raster.py:13-26 JIT-builds),
                             compiled from the reference tree for sm_100a by torch's extension builder into
                             that folder - a GPU comparator for the gs2d parity tests, loaded there as a
                             module from the built file (the reference tree is not on the GPU box)
  oracle/_ref/splat2d_cuda_ref/splat2d_cuda_ref.so   the reference's own splat2d extension with its CUDA
                             kernels (phase0/csrc/macrotile: bindings.cpp, splat2d_cpu.cpp, splat2d_fwd.cu,
                             splat2d_bwd_pixel.cu, splat2d_bwd_splat.cu, the sources and -DWITH_CUDA build of
                             phase0/splat2d/ops.py:33-45 with an sm_100a target), built the same way
  oracle/_ref/fastergs_macro/libfastergs_macro_ref.so   the reference's own Faster-GS blend backward
                             (blend_backward_macro_cu): its source exists only as the lines
                             phase1/fastergs_macro.patch adds to kernels_backward.cuh, which are extracted into
                             that folder and compiled for sm_100a with nvcc behind oracle/fastergs_macro_ref.cu,
                             under the names oracle/fastergs_ref_config.cuh supplies

The reference tree is found through --reference, the REFERENCE_ROOT environment variable, or a folder named
"reference" beside this repository's root; without one only liboracle.so is built.

Built files are git-ignored; they travel to the GPU box with the working tree.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
CXX = os.environ.get("ORACLE_CXX", "g++")  # the PATH g++ (the image's $CXX wrapper lacks libgomp)
FLAGS = ["-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math"]


def _compile(out: Path, sources: list[Path], flags: list[str], extra_inputs: list[Path] = ()) -> Path:
    inputs = list(sources) + list(extra_inputs)
    stamp = out.with_suffix(out.suffix + ".stamp")
    h = hashlib.sha256(" ".join(flags).encode())
    for p in inputs:
        h.update(p.read_bytes())
    digest = h.hexdigest()
    if out.exists() and stamp.exists() and stamp.read_text() == digest:
        return out
    cmd = [CXX, *flags, *map(str, sources), "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    stamp.write_text(digest)
    return out


def reference_root(arg: str | None = None) -> Path | None:
    root = arg or os.environ.get("REFERENCE_ROOT")
    if root is None:
        sibling = HERE.parent.parent / "reference"
        root = str(sibling) if sibling.is_dir() else None
    return Path(root) if root and Path(root).is_dir() else None


def build(reference: str | None = None) -> None:
    srcs = sorted(HERE.glob("*.cpp"))
    mine = [p for p in srcs if not p.name.endswith("_ref_capi.cpp")]
    if mine:
        _compile(HERE / "liboracle.so", mine, FLAGS + ["-fopenmp"], list(HERE.glob("*.h")))
    ref = reference_root(reference)
    if ref is not None:
        build_toy2d_cuda_ref(ref)
        build_splat2d_cuda_ref(ref)
        build_fastergs_macro_ref(ref)
        mt = ref / "phase0" / "csrc" / "macrotile"
        if (mt / "splat2d_cpu.cpp").exists():
            REF_OUT.mkdir(exist_ok=True)
            _compile(REF_OUT / "libsplat2d_ref.so", [HERE / "splat2d_ref_capi.cpp", mt / "splat2d_cpu.cpp"],
                     FLAGS + [f"-I{mt}"], [mt / "splat2d_common.h"])


TOY2D_REF_NAME = "gs2d_cuda_ref"


def build_toy2d_cuda_ref(ref: Path) -> Path | None:
    """The reference's toy2d CUDA extension, built for sm_100a into oracle/_ref/gs2d_cuda_ref (ninja keeps it
    current). Returns the built module file, or None when the reference's source is absent."""
    src = ref / "toy2d" / "csrc" / "rasterize.cu"
    if not src.exists():
        return None
    out_dir = REF_OUT / TOY2D_REF_NAME
    out_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    load(name=TOY2D_REF_NAME, sources=[str(src)], build_directory=str(out_dir),
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"], verbose=False)
    built = out_dir / f"{TOY2D_REF_NAME}.so"
    return built if built.exists() else None


SPLAT2D_REF_NAME = "splat2d_cuda_ref"


def build_splat2d_cuda_ref(ref: Path) -> Path | None:
    """The reference's splat2d extension with CUDA, built for sm_100a into oracle/_ref/splat2d_cuda_ref."""
    mt = ref / "phase0" / "csrc" / "macrotile"
    names = ("splat2d_cpu.cpp", "bindings.cpp", "splat2d_fwd.cu", "splat2d_bwd_pixel.cu", "splat2d_bwd_splat.cu")
    if not all((mt / nm).exists() for nm in names):
        return None
    out_dir = REF_OUT / SPLAT2D_REF_NAME
    out_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    load(name=SPLAT2D_REF_NAME, sources=[str(mt / nm) for nm in names], build_directory=str(out_dir),
         extra_cflags=["-O2", "-DWITH_CUDA"],
         extra_cuda_cflags=["-O2", "-std=c++17", "-DWITH_CUDA", "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_include_paths=[str(mt)], with_cuda=True, verbose=False)
    built = out_dir / f"{SPLAT2D_REF_NAME}.so"
    return built if built.exists() else None


FASTERGS_MACRO_DIR = REF_OUT / "fastergs_macro"
FASTERGS_MACRO_LIB = FASTERGS_MACRO_DIR / "libfastergs_macro_ref.so"


def extract_added_lines(patch: Path, target: str) -> str:
    """The lines a unified diff adds to the file whose path ends with ``target`` (the '+' prefix removed)."""
    out, inside = [], False
    for line in patch.read_text().splitlines():
        if line.startswith("diff --git"):
            inside = line.endswith(target)
            continue
        if not inside or line.startswith("+++") or line.startswith("---"):
            continue
        if line.startswith("+"):
            out.append(line[1:])
    return "\n".join(out) + "\n"


def build_fastergs_macro_ref(ref: Path) -> Path | None:
    """The reference's blend_backward_macro_cu, extracted from phase1/fastergs_macro.patch and compiled for sm_100a
    into oracle/_ref/fastergs_macro/libfastergs_macro_ref.so (C entry point: oracle/fastergs_macro_ref.cu)."""
    patch = ref / "phase1" / "fastergs_macro.patch"
    if not patch.exists():
        return None
    FASTERGS_MACRO_DIR.mkdir(parents=True, exist_ok=True)
    kernel = extract_added_lines(patch, "rasterization/include/kernels_backward.cuh")
    if "blend_backward_macro_cu" not in kernel:
        raise RuntimeError("phase1/fastergs_macro.patch: blend_backward_macro_cu not found in its added lines")
    inc = FASTERGS_MACRO_DIR / "blend_backward_macro.inc"
    if not inc.exists() or inc.read_text() != kernel:
        inc.write_text(kernel)
    srcs = [HERE / "fastergs_macro_ref.cu", HERE / "fastergs_ref_config.cuh", inc]
    flags = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC", "-shared",
             f"-I{HERE}", f"-I{FASTERGS_MACRO_DIR}"]
    stamp = FASTERGS_MACRO_LIB.with_suffix(".so.stamp")
    h = hashlib.sha256(" ".join(flags).encode())
    for p in srcs:
        h.update(p.read_bytes())
    if FASTERGS_MACRO_LIB.exists() and stamp.exists() and stamp.read_text() == h.hexdigest():
        return FASTERGS_MACRO_LIB
    import shutil

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, *flags, str(HERE / "fastergs_macro_ref.cu"), "-o", str(FASTERGS_MACRO_LIB)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference blend backward build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    stamp.write_text(h.hexdigest())
    return FASTERGS_MACRO_LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference")
    a = ap.parse_args()
    build(a.reference)
    return 0


if __name__ == "__main__":
    sys.exit(main())
