"""Builds oracle/_ref/libref_hip.so: the reference's own HIP kernels compiled for the host — TEST INFRASTRUCTURE ONLY.

The four kernel sources of the reference (int8_gemm.hip, hip_attention.hip, int8_gemv.hip, rms_norm.hip) are read
from the reference checkout (environment variable REF_DIR, default the checkout's location on the build machine) and
compiled by g++ against the CPU stand-in for <hip/hip_runtime.h> in this directory. The one edit made to a source on
its way to the compiler is to its clang vector typedefs (`typedef T name __attribute__((ext_vector_type(N)))`, which
g++ does not know): each becomes `typedef hipemu::Vec<T, N> name`, a struct with the same elements, `.x`..`.w`
accessors and element-wise operators. The edited sources are written to oracle/_ref/ only for the compiler and
removed once compiled; oracle/_ref/ is not part of the repository.

Usage: python oracle/hipemu/build.py [--force]. Exits 0 without building when the reference checkout is absent.
"""
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE = os.path.dirname(HERE)
OUT = os.path.join(ORACLE, "_ref")
LIB = os.path.join(OUT, "libref_hip.so")
SOURCES = ["int8_gemm.hip", "hip_attention.hip", "int8_gemv.hip", "rms_norm.hip"]
# No contraction (the stand-in's rounding model); fp16 arithmetic rounds per operation; no type-based aliasing
# assumptions (the kernels reinterpret fp16 arrays as vectors).
CXXFLAGS = ["-std=c++20", "-O2", "-fPIC", "-ffp-contract=off", "-fexcess-precision=16", "-fno-strict-aliasing",
            "-fvisibility=hidden", "-w", "-I", HERE]
TYPEDEF = re.compile(r"typedef\s+(\w+)\s+(\w+)\s+__attribute__\(\(ext_vector_type\((\d+)\)\)\);")


def ref_dir():
    return os.environ.get("REF_DIR", "/root/reference")


def translate(text):
    out, n = TYPEDEF.subn(lambda m: f"typedef hipemu::Vec<{m.group(1)}, {m.group(3)}> {m.group(2)};", text)
    if n == 0:
        raise RuntimeError("no ext_vector_type typedef found: the source layout changed")
    return out


def build(force=False):
    src_dir = ref_dir()
    if not all(os.path.isfile(os.path.join(src_dir, s)) for s in SOURCES):
        print(f"reference kernel sources not found in {src_dir}; oracle/_ref not built")
        return None
    os.makedirs(OUT, exist_ok=True)
    deps = [os.path.join(src_dir, s) for s in SOURCES] + [os.path.join(HERE, f) for f in
                                                           ("runtime.cpp", "launch.cpp", "hipemu_core.h", "build.py",
                                                            os.path.join("hip", "hip_runtime.h"))]
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(d) for d in deps):
        return LIB
    objs = []
    for name in SOURCES:
        with open(os.path.join(src_dir, name)) as f:
            text = translate(f.read())
        cpp = os.path.join(OUT, name.replace(".hip", ".gen.cpp"))
        with open(cpp, "w") as f:
            f.write(text)
        obj = cpp.replace(".gen.cpp", ".o")
        try:
            subprocess.run(["g++", *CXXFLAGS, "-c", cpp, "-o", obj], check=True)
        finally:
            os.remove(cpp)
        objs.append(obj)
    for name in ("runtime.cpp", "launch.cpp"):
        obj = os.path.join(OUT, name.replace(".cpp", ".o"))
        subprocess.run(["g++", *CXXFLAGS, "-c", os.path.join(HERE, name), "-o", obj], check=True)
        objs.append(obj)
    subprocess.run(["g++", "-shared", "-o", LIB, *objs, "-lpthread"], check=True)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
