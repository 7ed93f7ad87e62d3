#!/usr/bin/env python3
"""Build oracle/_ref: the reference's own code, compiled here, used to pin the
CPU restatement (oracle/tmnn_oracle.c).  TEST INFRASTRUCTURE ONLY.

What is built (all from the reference sources where they lie; nothing is
copied into this repository):
  _ref/gen_msl                 the reference's KernelCompiler/MLPKernelEmitter
  _ref/libtmnn_ref_host.so     morton_sort.h, kernel_spec.cpp, adam_params.h
  _ref/libtmnn_ref_<tag>.so    the scalar train / external-grad / eval MSL the
                               emitter generates for spec <tag> (and its
                               simdgroup-matrix train kernel where the
                               compiler realises one), compiled as C++
                               through oracle/ref/metal_shim.h
  _ref/libtmnn_ref_static.so   the static Adam MSL (adam_kernel_msl.h) and the
                               Philox init MSL (metal_context.cpp)

Needs /root/reference (present in the build container only); the GPU box uses
the prebuilt files.  Usage: python oracle/ref_build.py [--force]
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF = os.environ.get("TMNN_REFERENCE_ROOT", "/root/reference")
def _find_nlohmann():
    """Directory holding nlohmann/json.hpp: TMNN_NLOHMANN_INCLUDE, else the
    copy cudnn-frontend vendors in the Python environment, else the system
    include path."""
    env = os.environ.get("TMNN_NLOHMANN_INCLUDE")
    if env:
        return env
    import sysconfig
    for base in {sysconfig.get_paths()["purelib"], sysconfig.get_paths()["platlib"]}:
        cand = os.path.join(base, "include", "cudnn_frontend", "thirdparty")
        if os.path.exists(os.path.join(cand, "nlohmann", "json.hpp")):
            return cand
    return "/usr/include"


NLOHMANN = _find_nlohmann()
CXX = ["g++", "-std=c++23", "-O2", "-fPIC", "-ffp-contract=off",
       "-Wno-attributes", "-w"]

# tag: (L, F, log2T, d, W, H, O, loss, base, scale, huber)
SPECS = {
    "ka": (2, 2, 10, 3, 8, 1, 1, 0, 4.0, 2.0, 1.0),
    "sdf": (8, 2, 12, 3, 16, 1, 1, 1, 16.0, 1.447, 1.0),
    "img": (4, 2, 12, 3, 16, 2, 3, 0, 16.0, 1.5, 1.0),
    "d4": (4, 2, 12, 4, 16, 2, 4, 0, 8.0, 1.5, 1.0),
    "d4o1": (4, 2, 12, 4, 16, 2, 1, 0, 8.0, 1.5, 1.0),
    "f1": (4, 1, 10, 3, 16, 1, 1, 2, 4.0, 2.0, 0.1),
    "f4": (4, 4, 10, 3, 16, 2, 1, 0, 4.0, 2.0, 1.0),
    "h3": (2, 2, 10, 3, 8, 3, 1, 0, 4.0, 2.0, 1.0),
    "cos": (4, 2, 10, 3, 16, 1, 3, 3, 4.0, 1.5, 1.0),
    # bench.py reference arm workloads
    "bench_sdf3d": (16, 2, 19, 3, 64, 1, 1, 1, 16.0, 1.447, 1.0),
    "bench_image": (16, 2, 15, 3, 64, 2, 3, 0, 16.0, 1.5, 1.0),
    "bench_field4d": (16, 2, 22, 4, 64, 2, 4, 0, 8.0, 1.5, 1.0),
}


def float_literals(msl):
    """Metal has no double: an unsuffixed literal such as `1.0` is a float.
    Compiled as C++ it would be a double and promote the expression around it,
    so give every unsuffixed decimal literal an `f` suffix."""
    return re.sub(r"(?<![\w.])(\d+\.\d*)(?![\w.])", r"\1f", msl)


def threadgroup_qualifiers(msl):
    """The shim maps `threadgroup` to `static`, which is right for the
    arrays a kernel body declares (one threadgroup runs at a time) but not
    for threadgroup pointers or array parameters (the SIMD training kernel
    passes its activation tiles to helpers): there the qualifier is dropped."""
    out, i = [], 0
    for m in re.finditer(r"\bthreadgroup\b(?!_)", msl):
        rest = msl[m.end():]
        stop = re.search(r"[;,)]", rest)
        stmt = rest[:stop.start()] if stop else rest
        body_array = stop and stop.group() == ";" and "=" not in stmt and "[" in stmt
        out.append(msl[i:m.start()])
        out.append("threadgroup" if body_array else "")
        i = m.end()
    out.append(msl[i:])
    return "".join(out)


def run(cmd, **kw):
    subprocess.run(cmd, check=True, **kw)


def newer(target, *deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False):
    if not os.path.isdir(REF):
        print(f"ref_build: {REF} absent; using prebuilt oracle/_ref",
              file=sys.stderr)
        return False
    os.makedirs(OUT, exist_ok=True)
    inc = ["-I" + os.path.join(REF, "include"), "-I" + os.path.join(REF, "src"),
           "-I" + NLOHMANN]
    kdir = os.path.join(REF, "src/tiny_metal_nn/kernels")
    gen = os.path.join(OUT, "gen_msl")
    if force or newer(gen, os.path.join(HERE, "ref/gen_msl.cpp")):
        run(CXX + inc + [os.path.join(HERE, "ref/gen_msl.cpp"),
                         os.path.join(kdir, "kernel_compiler.cpp"),
                         os.path.join(kdir, "kernel_spec.cpp"),
                         os.path.join(kdir, "mlp_kernel_emitter.cpp"),
                         "-o", gen])
    host = os.path.join(OUT, "libtmnn_ref_host.so")
    if force or newer(host, os.path.join(HERE, "ref/ref_host.cpp")):
        run(CXX + ["-shared"] + inc + [os.path.join(HERE, "ref/ref_host.cpp"),
                                       os.path.join(kdir, "kernel_spec.cpp"),
                                       "-o", host])
    shim = ["-I" + os.path.join(HERE, "ref"),
            "-I" + os.path.join(HERE, "ref/include")]
    drv = os.path.join(HERE, "ref/ref_kernels.cpp")
    rt = os.path.join(HERE, "ref/shim_rt.cpp")
    deps = [drv, rt, os.path.join(HERE, "ref/metal_shim.h"), gen]
    for tag, sp in SPECS.items():
        so = os.path.join(OUT, f"libtmnn_ref_{tag}.so")
        if not (force or newer(so, *deps)):
            continue
        args = [str(x) for x in sp]
        objs = []
        roles = [("train", "ROLE_TRAIN"), ("extgrad", "ROLE_EXTGRAD"),
                 ("eval", "ROLE_EVAL")]
        if sp[6] == 1:  # the EvalGradient kernel is single-output
            roles.append(("evalgrad", "ROLE_EVALGRAD"))
        # the simdgroup-matrix training kernel, for the shapes where the
        # reference's compiler realises it (its default there)
        probe = subprocess.run([gen, "train"] + args + ["1", "1"], check=True,
                               capture_output=True, text=True)
        simd = "simd=1" in probe.stderr
        if simd:
            roles.append(("train_simd", "ROLE_TRAIN_SIMD"))
        # bench.py's reference arm: the scalar training kernel with
        # threadgroups running concurrently on the host cores
        if tag.startswith("bench_"):
            roles.append(("train_lanes", "ROLE_TRAIN_LANES"))
        for role, define in roles:
            msl = os.path.join(OUT, f"{tag}_{role}.msl")
            gen_role = "train" if role in ("train_simd", "train_lanes") else role
            flags = ["0" if role.startswith("eval") else "1"]
            if role == "train_simd":
                flags.append("1")
            text = subprocess.run([gen, gen_role] + args + flags, check=True,
                                  capture_output=True, text=True).stdout
            with open(msl, "w") as f:
                f.write(threadgroup_qualifiers(float_literals(text)))
            obj = os.path.join(OUT, f"{tag}_{role}.o")
            run(CXX + shim + ["-c", drv, f"-D{define}",
                              f'-DMSL_FILE="{msl}"', "-o", obj])
            objs.append(obj)
        run(CXX + ["-shared"] + shim + objs + [rt, "-o", so, "-lpthread"])
    # static MSL: Adam (header string constants) and Philox init (raw string
    # literals inside metal_context.cpp, extracted verbatim at build time).
    so = os.path.join(OUT, "libtmnn_ref_static.so")
    if force or newer(so, *deps):
        hdr = os.path.join(REF, "include/tiny-metal-nn/kernels/adam_kernel_msl.h")
        text = open(hdr).read()
        lits = re.findall(r'R"msl\((.*?)\)msl"', text, re.S)
        adam = os.path.join(OUT, "static_adam.msl")
        with open(adam, "w") as f:
            f.write("#define USE_INT_ATOMICS_HASH\n")
            f.write("#define SPARSE_HASH_ENTRY_WIDTH 2u\n")
            for lit in lits:
                f.write(lit + "\n")
        ctx = open(os.path.join(REF, "src/tiny_metal_nn/runtime/metal_context.cpp")).read()
        msls = re.findall(r'R"MSL\((.*?)\)MSL"', ctx, re.S)
        objs = []
        for name, body, define in (("adam", None, "ROLE_ADAM"),
                                   ("init", msls[0], "ROLE_INIT"),
                                   ("normal", msls[1], "ROLE_NORMAL")):
            msl = adam if body is None else os.path.join(OUT, f"static_{name}.msl")
            if body is not None:
                with open(msl, "w") as f:
                    f.write(body)
            obj = os.path.join(OUT, f"static_{name}.o")
            run(CXX + shim + ["-c", drv, f"-D{define}", f'-DMSL_FILE="{msl}"',
                              "-o", obj])
            objs.append(obj)
        run(CXX + ["-shared"] + shim + objs + [rt, "-o", so, "-lpthread"])
    return True


if __name__ == "__main__":
    build(force="--force" in sys.argv)
