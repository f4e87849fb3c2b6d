"""Builds libsjk_b200.so in place (sm_100a) from csrc/. Used by __graft_entry__.build() and the tests.

    python build.py            # build if any source is newer than the library
    python build.py --force    # rebuild
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsjk_b200.so")
OBJDIR = os.path.join(HERE, "_build")
SOURCES = ["sjk_stage.cu", "sjk_seal.cu", "sjk_decode.cu", "sjk_attend.cu", "sjk_attend_tc.cu", "sjk_attend_dense.cu",
           "sjk_attend_trellis.cu", "sjk_attend_batch.cu", "sjk_synth.cu", "sjk_xchg.cu", "sjk_pool.cu", "sjk_host.cpp"]
HEADERS = ["sjk_common.cuh", "sjk_internal.h", "sjk_tables.h", "sjk_tc.cuh", "sjk_desc.cuh", "sjk_plan.cuh", "sjk_synth.h", "sjk_merge.cuh", "sjk_fwht.cuh", "../../include/sjk.h"]
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _stale(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, h) for h in HEADERS]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    os.makedirs(OBJDIR, exist_ok=True)
    objs, procs = [], []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJDIR, s + ".o")
        objs.append(obj)
        if force or _stale(obj, src):
            cmd = [NVCC] + ARCH + FLAGS + ["-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for s, p in procs:
        out = p.communicate()[0].decode()
        if p.returncode != 0:
            failed.append((s, out))
        elif verbose and out.strip():
            print(out)
    if failed:
        for s, out in failed:
            sys.stderr.write(f"--- {s}\n{out}\n")
        raise RuntimeError("nvcc failed: " + ", ".join(s for s, _ in failed))
    if force or procs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
