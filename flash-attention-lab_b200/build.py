"""Builds libflash_lab_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python flash-attention-lab_b200/build.py [--force] [--debug]

Every .cu / .cpp under csrc/ is compiled with
    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -std=c++17 -Xptxas -v
and linked into flash_lab/libflash_lab_b200.so next to the Python package that loads it. The
ptxas resource report (registers, spills, shared memory per kernel) goes to
build/ptxas.txt. Rebuilds only when a source, header or this script is newer than the library.

Then binding/torch_ops.cpp (host C++, no kernels) is compiled against PyTorch's headers with
torch.utils.cpp_extension into flash_lab/_flash_lab_torch.so, linked to the library above: the
binding flash_lab.ops uses for eager calls (ATen allocation + the C ABI, without ctypes).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
BUILD = HERE / "build"
LIB = HERE / "flash_lab" / "libflash_lab_b200.so"
BINDING_SRC = HERE / "binding" / "torch_ops.cpp"
BINDING = HERE / "flash_lab" / "_flash_lab_torch.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
          "-I", str(CSRC), "--expt-relaxed-constexpr"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources() -> list[pathlib.Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def needs_rebuild() -> bool:
    if not LIB.exists():
        return True
    stamp = LIB.stat().st_mtime
    deps = [*sources(), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h"),
            pathlib.Path(__file__)]
    return any(p.stat().st_mtime > stamp for p in deps)


def compile_one(src: pathlib.Path, debug: bool, defines=(), build_dir=None):
    obj = (build_dir or BUILD) / (src.name + ".o")
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"]
    if debug:
        cmd += ["-DFLB_DEBUG=1"]
    cmd += [f"-D{d}" for d in defines]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, debug: bool = False, verbose: bool = False, defines=(),
          out: pathlib.Path | None = None) -> pathlib.Path:
    """Builds the library (to `out` with extra -D `defines` for instrumented variants)."""
    lib = out or LIB
    if not force and out is None and not needs_rebuild():
        return LIB
    build_dir = BUILD if out is None else pathlib.Path(str(out) + ".build")
    build_dir.mkdir(exist_ok=True, parents=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        results = list(pool.map(lambda s: compile_one(s, debug, defines, build_dir), srcs))
    report = "\n".join(f"== {src.name}\n{log}" for src, (_, log) in zip(srcs, results))
    (build_dir / "ptxas.txt").write_text(report)
    if verbose:
        print(report)
    tmp = lib.with_suffix(".so.tmp")
    # The CUDA runtime is linked statically; driver entry points (cuTensorMapEncodeTiled) are
    # resolved at run time through cudaGetDriverEntryPoint, so the library loads without a GPU.
    cmd = [nvcc(), *ARCH, "-shared", "-Xlinker", f"-soname={LIB.name}", "-o", str(tmp),
           *[str(o) for o, _ in results]]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, lib)
    return lib


def build_binding(force: bool = False) -> pathlib.Path:
    """Compiles the PyTorch binding (binding/torch_ops.cpp) against the built library."""
    deps = [BINDING_SRC, *INCLUDE.glob("*.h"), LIB, pathlib.Path(__file__)]
    if not force and BINDING.exists() and all(d.stat().st_mtime <= BINDING.stat().st_mtime
                                             for d in deps):
        return BINDING
    import ctypes

    from torch.utils import cpp_extension

    # cpp_extension.load imports the module from the build folder: the library it needs is found
    # loaded already, by its SONAME (in the package, $ORIGIN finds it).
    ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)
    build_dir = BUILD / "torch_binding"
    build_dir.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name="_flash_lab_torch", sources=[str(BINDING_SRC)], build_directory=str(build_dir),
        extra_include_paths=[str(INCLUDE)], with_cuda=True,
        extra_cflags=["-O2", "-std=c++17"],
        # Ninja turns "$$" into "$" and its shell keeps the backslashed "$": the runpath is a
        # literal $ORIGIN, so the binding finds the library in its own folder.
        extra_ldflags=[f"-L{LIB.parent}", "-lflash_lab_b200", "-Wl,-rpath,\\$$ORIGIN"],
        verbose=False)
    built = build_dir / "_flash_lab_torch.so"
    tmp = BINDING.with_suffix(".so.tmp")
    shutil.copyfile(built, tmp)
    os.replace(tmp, BINDING)
    return BINDING


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("-D", dest="defines", action="append", default=[],
                    help="extra preprocessor define (instrumented builds, e.g. FLB_PREFILL_TRACE)")
    ap.add_argument("--out", type=pathlib.Path, default=None, help="library path for a variant")
    args = ap.parse_args()
    lib = build(force=args.force, debug=args.debug, verbose=args.verbose, defines=args.defines,
                out=args.out)
    print(lib)
    if args.out is None:
        print(build_binding(force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
