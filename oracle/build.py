"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles the C restatement ``lh_oracle.c`` into
  ``oracle/_ref/liblh_oracle.so``.
* ``build_ref()`` renders the reference's own selection kernel source from
  ``src/lighthouse_selection_cuda.py:7-331`` (the ``_make_kernel_source``
  function, called here, never copied) for pooling factors 2, 4 and 8 and
  compiles it twice:

  - as C++ on host threads (``ref_cpu_shim.h``) ->
    ``oracle/_ref/libref_cpu_p{p}.so``: the reference kernel itself running on
    the CPU, used to pin the C restatement and to make golden vectors;
  - with nvcc for sm_100a and the reference's NVRTC flags (``--use_fast_math``)
    -> ``oracle/_ref/libref_gpu_p{p}.so``: the reference kernel on the GPU,
    used by the GPU parity tests.

  The rendered ``.cu`` text is written to ``oracle/_ref/`` (git-ignored) only
  for the compile and deleted afterwards.  ``build_ref()`` needs the reference
  tree and therefore only runs in the build container; the built ``.so`` files
  travel with the repository snapshot to the GPU box.

Nothing in the product package imports this module.
"""
from __future__ import annotations

import importlib.util
import os
import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
# The reference tree: LH_REFERENCE_ROOT, else the build container's mount point.
REFERENCE_ROOT = pathlib.Path(os.environ.get("LH_REFERENCE_ROOT", "/root/reference"))
REFERENCE_CU = REFERENCE_ROOT / "src" / "lighthouse_selection_cuda.py"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
POOLING_FACTORS = (2, 4, 8)


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True, cwd=HERE)


def build_oracle() -> pathlib.Path:
    OUT.mkdir(exist_ok=True)
    so = OUT / "liblh_oracle.so"
    src = HERE / "lh_oracle.c"
    if not so.exists() or so.stat().st_mtime < src.stat().st_mtime:
        _run(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-o", str(so), str(src)])
    return so


def _render_reference_source(pf: int) -> str:
    spec = importlib.util.spec_from_file_location("_lh_reference_selection_cuda", REFERENCE_CU)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod._make_kernel_source(pf, 128)


def build_ref(force: bool = False, gpu: bool = True) -> list[pathlib.Path]:
    """Compile the reference kernel for CPU (and GPU). Returns built paths."""
    if not REFERENCE_CU.exists():
        return []
    OUT.mkdir(exist_ok=True)
    built = []
    for pf in POOLING_FACTORS:
        cpu_so = OUT / f"libref_cpu_p{pf}.so"
        gpu_so = OUT / f"libref_gpu_p{pf}.so"
        need_cpu = force or not cpu_so.exists()
        need_gpu = gpu and (force or not gpu_so.exists())
        if not (need_cpu or need_gpu):
            built += [cpu_so] + ([gpu_so] if gpu else [])
            continue
        src = OUT / f"ref_topk_p{pf}.cu"
        src.write_text(_render_reference_source(pf))
        try:
            if need_cpu:
                _run(["g++", "-O2", "-std=c++20", "-shared", "-fPIC", "-pthread",
                      f'-DREF_SRC="{src}"', "-o", str(cpu_so), str(HERE / "ref_cpu_launch.cpp")])
            if need_gpu:
                _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "--use_fast_math",
                      "-std=c++17", "-O3", "-shared", "-Xcompiler", "-fPIC",
                      f'-DREF_SRC="{src}"', "-o", str(gpu_so), str(HERE / "ref_gpu_launch.cu")])
        finally:
            src.unlink(missing_ok=True)
        built += [cpu_so] + ([gpu_so] if gpu else [])
    return built


if __name__ == "__main__":
    print(build_oracle())
    for p in build_ref():
        print(p)
