"""Builds libgptb200.so (the sm_100a kernels + the C ABI) in-tree.

Every `.cu` / `.cpp` file under csrc/ is compiled by nvcc for sm_100a only and
linked into rig_b200/libgptb200.so next to the Python front-end, so the shared
object travels with the source tree. Objects are rebuilt only when a source or
header is newer than the object.
"""

from __future__ import annotations

import concurrent.futures
import os
import re
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT_DIR = HERE / "rig_b200"
LIB = OUT_DIR / "libgptb200.so"
OBJ_DIR = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "-I",
    str(INCLUDE),
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libgptb200")
    return cand


def _sources() -> list[pathlib.Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers_mtime() -> float:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".cuh", ".h")]
    hs += list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in hs), default=0.0)


def _compile(src: pathlib.Path, force: bool) -> pathlib.Path:
    obj = OBJ_DIR / (src.name + ".o")
    if not force and obj.exists():
        newest = max(src.stat().st_mtime, _headers_mtime())
        if obj.stat().st_mtime >= newest:
            return obj
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = True) -> pathlib.Path:
    OBJ_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if LIB.exists() and not force:
        if LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
            return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


def ptxas_report(dest: pathlib.Path) -> None:
    """Compiles every CUDA source once more with `-Xptxas -v` and writes, per
    kernel instantiation, the registers per thread, spill bytes, stack frame and
    static shared memory ptxas reports (one line each, names demangled)."""

    import tempfile

    rows = []
    with tempfile.TemporaryDirectory() as tmp:
        for src in _sources():
            cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-c", str(src),
                   "-o", str(pathlib.Path(tmp) / (src.name + ".o"))]
            if src.suffix == ".cpp":
                cmd[1:1] = ["-x", "cu"]
            log = subprocess.run(cmd, check=True, capture_output=True, text=True).stderr
            name, props = None, {}
            for line in log.splitlines():
                m = re.search(r"Function properties for (\S+)", line)
                if m:
                    name, props = m.group(1), {}
                    continue
                m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
                if m and name:
                    props.update(stack=int(m.group(1)), spill_st=int(m.group(2)), spill_ld=int(m.group(3)))
                    continue
                m = re.search(r"Used (\d+) registers", line)
                if m and name:
                    smem = re.search(r"(\d+) bytes smem", line)
                    rows.append((src.name, name, int(m.group(1)), props.get("spill_st", 0),
                                 props.get("spill_ld", 0), props.get("stack", 0),
                                 int(smem.group(1)) if smem else 0))
                    name = None
    filt = shutil.which("c++filt")
    names = [r[1] for r in rows]
    if filt:
        out = subprocess.run([filt], input="\n".join(names), capture_output=True, text=True, check=True)
        names = out.stdout.splitlines()
    lines = ["# ptxas resource usage of libgptb200 (sm_100a, -O3)", "",
             "Command: python gpt-speedrun-tpu_b200/build.py --ptxas-report", "",
             "file | registers/thread | spill stores B | spill loads B | stack B | static smem B | kernel",
             "---|---|---|---|---|---|---"]
    for (src, _m, regs, sst, sld, stk, smem), nm in zip(rows, names):
        nm = re.sub(r"\s+", " ", nm)[:160]
        lines.append(f"{src} | {regs} | {sst} | {sld} | {stk} | {smem} | `{nm}`")
    dest.write_text("\n".join(lines) + "\n")
    print(f"wrote {dest} ({len(rows)} kernels)")


if __name__ == "__main__":
    if "--ptxas-report" in sys.argv:
        ptxas_report(HERE.parent / "profiles" / "ptxas_resource_usage.md")
    else:
        build(force="--force" in sys.argv)
