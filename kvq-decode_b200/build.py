"""Build the bpt CUDA library in-tree: kvq-decode_b200/bpt/libbpt_b200.so.

    python kvq-decode_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
with nvcc and links one shared library exporting the C ABI declared in ``include/bpt.h``.
The CUDA runtime is linked statically; the driver API is reached through
``cudaGetDriverEntryPointByVersion`` so the library has no link-time libcuda dependency.
Rebuilds only when a source or header is newer than the library.
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "bpt", "libbpt_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-O3"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return (sources() + glob.glob(os.path.join(CSRC, "*.cuh")) +
            glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(ROOT, "include", "*.h")) + [os.path.abspath(__file__)])


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in deps())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if not force and up_to_date():
        return OUT
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-c", src,
               "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for src, pr in procs:
        out, _ = pr.communicate()
        if pr.returncode != 0:
            failed.append((src, out))
        elif verbose and out.strip():
            print(out)
    if failed:
        msg = "\n".join(f"--- {s}\n{o}" for s, o in failed)
        raise RuntimeError("nvcc failed:\n" + msg)
    tmp = OUT + ".tmp"
    link = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-cudart",
            "static"]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    os.replace(tmp, OUT)
    return OUT


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose,
                extra=extra))


if __name__ == "__main__":
    sys.exit(main())
