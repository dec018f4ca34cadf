"""Build libmoek_b200.so in the package directory with nvcc for sm_100a (no GPU needed to build).

Variants (``variant``), each its own library next to the default one, selected at load time by ``MOEK_B200_LIB``:

- ``""``      libmoek_b200.so: the product.
- ``"trace"`` libmoek_b200_trace.so, built with -DMOEK_TRACE: the kernels also write %globaltimer stamps of their
              phases into a device array that ``moek_trace_read`` copies out (``qwen38_flash_coder_b200.trace``).
- ``"debug"`` libmoek_b200_debug.so, built with -DMOEK_DEBUG_CHECKS: the kernels also check every index they take
              from their inputs (sorted ids, expert ids, token rows, exception entries) before using it, record
              MOEK_DEV_BAD_INPUT in the device error word and skip the access instead of reading or writing out of
              bounds.

The sources compile in parallel (one nvcc per file) and link once.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
SOURCES = ["moek_abi.cu", "moek_align.cu", "moek_decode.cu", "moek_layer.cu", "moek_prefill.cu", "moek_ep.cu",
           "moek_router.cu", "moek_shared.cu", "moek_prep.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]
VARIANTS = {"": [], "trace": ["-DMOEK_TRACE"], "debug": ["-DMOEK_DEBUG_CHECKS"]}


def lib_path(variant: str = "") -> str:
    return os.path.join(HERE, "libmoek_b200" + (f"_{variant}" if variant else "") + ".so")


LIB = lib_path()


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def stale(variant: str = "") -> bool:
    lib = lib_path(variant)
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("moek_b200: nvcc failed: " + " ".join(cmd[-3:]))
    return r


def build(force: bool = False, verbose: bool = False, extra=(), variant: str = "") -> str:
    lib = lib_path(variant)
    if not force and not stale(variant):
        return lib
    objdir = os.path.join(HERE, "_build", variant or "default")
    os.makedirs(objdir, exist_ok=True)
    defs = VARIANTS[variant] + list(extra)
    objs = [os.path.join(objdir, s[:-3] + ".o") for s in SOURCES]
    cmds = [[nvcc()] + FLAGS + defs + ["-c", "-o", o, os.path.join(CSRC, s)]
            for s, o in zip(SOURCES, objs)]
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 4)) as ex:
        list(ex.map(lambda c: _run(c, verbose), cmds))
    _run([nvcc()] + ARCH + ["-shared", "-o", lib] + objs, verbose)
    return lib


def build_all(force: bool = False, verbose: bool = False):
    return [build(force=force, verbose=verbose, variant=v) for v in VARIANTS]


if __name__ == "__main__":
    args = [a for a in sys.argv[1:]]
    force = "--force" in args
    variants = [a.split("=", 1)[1] for a in args if a.startswith("--variant=")]
    extra = [a for a in args if a != "--force" and not a.startswith("--variant=")]
    if "--all" in args:
        extra.remove("--all")
        variants = list(VARIANTS)
    for v in variants or [""]:
        print(build(force=force, verbose=True, extra=extra, variant=v))
