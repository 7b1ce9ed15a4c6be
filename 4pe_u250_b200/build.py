"""Builds the native parts of the package in-tree.

  libi4d.so        the CUDA decode library (sm_100a) behind include/i4d.h
  libi4d_synth.so  seeded synthetic model images in the reference format
  i4d_decode       C++ host program over libi4d (replaces decode_host)
  csrc/gen/*       build-time tables (expf constants and exceptions)

Run as ``python -m`` or through ``__graft_entry__.build()``.  The expf
exception table is measured against this machine's C library once and
reused while its inputs are unchanged.
"""
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
GEN = os.path.join(CSRC, "gen")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd, cwd=None):
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=cwd)


def _digest(paths):
    h = hashlib.sha256()
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_expf_tables():
    os.makedirs(GEN, exist_ok=True)
    consts = os.path.join(GEN, "expf_consts.h")
    gen_py = os.path.join(CSRC, "gen_expf_consts.py")
    if _newer(consts, [gen_py]):
        _run([sys.executable, gen_py, consts])
    impl = os.path.join(CSRC, "i4d_expf_impl.h")
    tool_src = os.path.join(CSRC, "gen_expf_table.c")
    table = os.path.join(GEN, "expf_fix_table.c")
    stamp = os.path.join(GEN, "expf_fix_table.sha256")
    key = _digest([consts, impl, tool_src])
    if os.path.exists(table) and os.path.exists(stamp) and open(stamp).read().strip() == key:
        return table
    tool = os.path.join(GEN, "gen_expf_table")
    _run(["gcc", "-O2", "-mfma", "-ffp-contract=off", "-fopenmp", "-I", CSRC, tool_src, "-o", tool, "-lm"])
    _run([tool, table])
    with open(stamp, "w") as f:
        f.write(key + "\n")
    return table


def build_synth():
    src = os.path.join(CSRC, "synth.c")
    out = os.path.join(HERE, "libi4d_synth.so")
    if _newer(out, [src]):
        _run(["gcc", "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", src, "-o", out, "-lm"])
    return out


def build_i4d():
    table = build_expf_tables()
    srcs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    srcs.append(os.path.join(ROOT, "include", "i4d.h"))
    out = os.path.join(HERE, "libi4d.so")
    if not _newer(out, srcs + [table]):
        return out
    obj_dir = os.path.join(ROOT, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    cu_obj = os.path.join(obj_dir, "i4d.o")
    tab_obj = os.path.join(obj_dir, "expf_fix_table.o")
    _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-Xptxas", "-v",
          "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
          "-c", os.path.join(CSRC, "i4d.cu"), "-o", cu_obj])
    _run(["gcc", "-O1", "-fPIC", "-c", table, "-o", tab_obj])
    _run([NVCC, *ARCH, "-shared", "-o", out, cu_obj, tab_obj])
    return out


def build_host():
    src = os.path.join(CSRC, "host", "i4d_decode.cpp")
    out = os.path.join(HERE, "i4d_decode")
    lib = os.path.join(HERE, "libi4d.so")
    if _newer(out, [src, lib, os.path.join(ROOT, "include", "i4d.h")]):
        _run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), src, "-o", out,
              "-L" + HERE, "-l:libi4d.so", "-Wl,-rpath,$ORIGIN"])
    return out


def build_oracle():
    """The C restatement always; the reference emulator (oracle/_ref) only
    where I4D_REF_ROOT names a reference tree."""
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"])
    ref_root = os.environ.get("I4D_REF_ROOT")
    if ref_root and os.path.isdir(ref_root):
        _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", "REF_ROOT=" + ref_root])


def main():
    build_synth()
    build_i4d()
    build_host()
    build_oracle()


if __name__ == "__main__":
    main()
