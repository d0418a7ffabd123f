"""Build recipe of the reference-kernel oracle ``oracle/_ref/libervf_ref.so``.

TEST INFRASTRUCTURE.  kennydd001/ervf keeps its CUDA kernels as Python
string literals and compiles them at run time (CuPy RawModule / NVRTC,
fused_nvfp4.py:756, gpu_kernels.py:1525).  This recipe reads those literals
with ``ast`` from the reference tree where it lies (no import, no CuPy),
writes them under ``oracle/_ref/`` (git-ignored) and compiles them for
sm_100a with the reference's own options (``-std=c++14``; ``--use_fast_math``
for gpu_kernels, as at gpu_kernels.py:1525) together with the launchers in
``oracle/ref_launch.cu``.  The built library travels to the GPU box; the
reference tree itself is only needed here.

Sources used:
  src/moe_lab/lightningstream_nemotron/fused_nvfp4.py        _KERNEL_SOURCE
  scripts/nervf_nemotron/nervf01_geometry_audit.py           _ERVF_TEMPLATE (W = 4, 8, 32)
  src/moe_lab/lightningstream_nemotron/gpu_kernels.py        _SOURCE (gemv_bf16, gemv_f32)
  src/moe_lab/lightningstream_nemotron/sweepspec.py          _SOURCE (SweepMoE's batched kernels)
"""

from __future__ import annotations

import ast
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libervf_ref.so"
# The kennydd001/ervf checkout: $ERVF_REFERENCE, else a directory named
# `reference` beside this repository's root.
REF = Path(os.environ.get("ERVF_REFERENCE") or HERE.parent.parent / "reference")

FILES = {
    "fused": ("src/moe_lab/lightningstream_nemotron/fused_nvfp4.py", "_KERNEL_SOURCE"),
    "ervf": ("scripts/nervf_nemotron/nervf01_geometry_audit.py", "_ERVF_TEMPLATE"),
    "gpu": ("src/moe_lab/lightningstream_nemotron/gpu_kernels.py", "_SOURCE"),
    "sweep": ("src/moe_lab/lightningstream_nemotron/sweepspec.py", "_SOURCE"),
}
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def literal(path: Path, name: str) -> str:
    tree = ast.parse(path.read_text(encoding="utf-8"))
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id == name for t in node.targets):
            return ast.literal_eval(node.value)
    raise KeyError(f"{name} not found in {path}")


def available() -> bool:
    return all((REF / rel).exists() for rel, _ in FILES.values())


def build(force: bool = False) -> Path | None:
    if LIB.exists() and not force:
        return LIB
    if not available():
        return None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.mkdir(exist_ok=True)
    (OUT / "ref_fused.cu").write_text(literal(REF / FILES["fused"][0], FILES["fused"][1]))
    tmpl = literal(REF / FILES["ervf"][0], FILES["ervf"][1])
    for w in (4, 8, 32):
        (OUT / f"ref_ervf_w{w}.cu").write_text(tmpl.replace("__W__", str(w)))
    (OUT / "ref_gpu_kernels.cu").write_text(literal(REF / FILES["gpu"][0], FILES["gpu"][1]))
    (OUT / "ref_sweep.cu").write_text(literal(REF / FILES["sweep"][0], FILES["sweep"][1]))

    launch = HERE / "ref_launch.cu"
    units = [("fused", ["-DREF_FUSED", "-std=c++14"]),
             ("gpu", ["-DREF_GPU_KERNELS", "-std=c++14", "--use_fast_math"]),
             ("sweep", ["-DREF_SWEEP", "-std=c++14"])]
    for w in (4, 8, 32):
        units.append((f"ervf_w{w}", ["-DREF_ERVF_W=%d" % w, "-std=c++14",
                                     f"-DREF_KERNEL_NAME=ref_kernel_ervf_w{w}",
                                     f"-DREF_LAUNCH_NAME=ref_gemv_ervf_w{w}",
                                     f'-DREF_ERVF_FILE="ref_ervf_w{w}.cu"']))
    objs = []
    for tag, flags in units:
        obj = OUT / f"ref_{tag}.o"
        cmd = [nvcc, *ARCH, "-O3", "-Xcompiler", "-fPIC,-fvisibility=hidden", f"-I{OUT}", *flags,
               "-c", str(launch), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".tmp")
    subprocess.run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
