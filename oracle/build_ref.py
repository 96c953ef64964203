"""TEST INFRASTRUCTURE ONLY: compile the reference's own CPU op from its sources.

Builds ``streamtopk_sae_native`` (CPU entry ``streamtopk_cpu_forward`` only)
from the two reference source files where they lie:

    <ref>/streamtopk_sae/csrc/bindings.cpp           (pybind module, WITH_CUDA unset)
    <ref>/streamtopk_sae/csrc/cpu/streamtopk_cpu.cpp (process_row / dispatch_rows)

with the reference's C++ flags (``setup.py:15-28``: -O3 -ffast-math), except
that ``-march=native`` becomes ``-march=x86-64-v3`` so the object built here
also runs on the GPU box's host CPU.  Output goes only to ``oracle/_ref/``
(git-ignored; it travels to the GPU box with the snapshot).  No reference
source is copied into this repository.

With ``--cuda`` it also builds the reference's CUDA op
(``streamtopk_cuda_exact_forward`` / ``streamtopk_cuda_approx_forward``) as the
module ``streamtopk_sae_native_cuda`` in ``oracle/_ref/cuda/``: the same four
sources and flags as the reference's ``setup.py:15-38`` (``WITH_CUDA``,
nvcc -O3 --use_fast_math -lineinfo), with ``-gencode arch=compute_100a,
code=sm_100a`` in place of its sm_80/86/89 list (it ships no PTX, so its own
build cannot run on B200).  Only the GPU comparison test loads it.

Usage: python oracle/build_ref.py --ref <reference tree> [--cuda]   (or STK_REFERENCE_ROOT=<reference tree>)
"""
import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_root: str, verbose: bool = False) -> str:
    csrc = os.path.join(ref_root, "streamtopk_sae", "csrc")
    sources = [os.path.join(csrc, "bindings.cpp"),
               os.path.join(csrc, "cpu", "streamtopk_cpu.cpp")]
    for s in sources:
        if not os.path.isfile(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT, exist_ok=True)
    from torch.utils.cpp_extension import load
    build_dir = os.path.join(OUT, "build")
    os.makedirs(build_dir, exist_ok=True)
    mod = load(name="streamtopk_sae_native", sources=sources,
               extra_include_paths=[csrc],
               extra_cflags=["-O3", "-march=x86-64-v3", "-ffast-math"],
               build_directory=build_dir, verbose=verbose, with_cuda=False)
    so = mod.__file__
    dst = os.path.join(OUT, os.path.basename(so))
    if os.path.abspath(so) != os.path.abspath(dst):
        shutil.copy2(so, dst)
    return dst


def build_cuda(ref_root: str, verbose: bool = False) -> str:
    csrc = os.path.join(ref_root, "streamtopk_sae", "csrc")
    sources = [os.path.join(csrc, "bindings.cpp"),
               os.path.join(csrc, "cpu", "streamtopk_cpu.cpp"),
               os.path.join(csrc, "cuda", "streamtopk_exact.cu"),
               os.path.join(csrc, "cuda", "streamtopk_approx.cu")]
    for s in sources:
        if not os.path.isfile(s):
            raise FileNotFoundError(s)
    out = os.path.join(OUT, "cuda")
    build_dir = os.path.join(out, "build")
    os.makedirs(build_dir, exist_ok=True)
    from torch.utils.cpp_extension import load
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    mod = load(name="streamtopk_sae_native_cuda", sources=sources,
               extra_include_paths=[csrc],
               extra_cflags=["-O3", "-march=x86-64-v3", "-ffast-math", "-DWITH_CUDA"],
               extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", "-DWITH_CUDA",
                                  "-gencode=arch=compute_100a,code=sm_100a"],
               build_directory=build_dir, verbose=verbose, with_cuda=True)
    so = mod.__file__
    dst = os.path.join(out, os.path.basename(so))
    if os.path.abspath(so) != os.path.abspath(dst):
        shutil.copy2(so, dst)
    return dst


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("STK_REFERENCE_ROOT"),
                    help="root of the reference tree (default: $STK_REFERENCE_ROOT)")
    ap.add_argument("--cuda", action="store_true", help="also build the reference's CUDA op for sm_100a")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(a.ref):
        print(f"reference tree {a.ref!r} absent; skipping oracle/_ref build")
        return 0
    print(build(a.ref, a.v))
    if a.cuda:
        print(build_cuda(a.ref, a.v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
