"""Build recipes for the oracle — TEST INFRASTRUCTURE ONLY.

* ``build_oracle_lib()`` compiles the C restatement ``oracle/oracle.c`` into
  ``oracle/liboracle.so`` with gcc (OpenMP for the timed CPU baseline).
* ``build_reference_ops()`` compiles the reference's own swap operator from its two source
  files where they lie (``aegaeon/ops/ops.cpp`` and ``aegaeon/ops/swap.cu`` of the reference
  checkout, bound as ``aegaeon.ops`` by ``aegaeon/setup.py:52-54``) into ``oracle/_ref/`` with
  torch's extension builder, for sm_100a. Nothing of the reference is copied into this
  repository; the build only reads the sources in place. The resulting module is used by the
  GPU tests as a bit-exact pin for ``swap`` and must never be imported by the product.

Run ``python oracle/build.py`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_MODULE = "aegaeon_ref_ops"
# The reference checkout is expected beside this repository (``<parent>/reference/aegaeon/ops``);
# AEGAEON_REFERENCE_OPS names another location of the reference's ``aegaeon/ops`` directory.
REFERENCE_OPS_DIR = os.environ.get(
    "AEGAEON_REFERENCE_OPS",
    os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "aegaeon", "ops"))


def build_oracle_lib(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    if not force and os.path.exists(ORACLE_SO) and os.path.getmtime(ORACLE_SO) >= os.path.getmtime(src):
        return ORACLE_SO
    cmd = ["gcc", "-O3", "-fopenmp", "-shared", "-fPIC", "-std=c11", "-o", ORACLE_SO + ".tmp", src, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(ORACLE_SO + ".tmp", ORACLE_SO)
    return ORACLE_SO


def reference_ops_available() -> bool:
    return all(os.path.exists(os.path.join(REFERENCE_OPS_DIR, f)) for f in ("ops.cpp", "swap.cu", "ops.h"))


def build_reference_ops(verbose: bool = False) -> str | None:
    """Compile the reference swap op into oracle/_ref; returns the .so path or None."""
    if not reference_ops_available():
        return None
    so = os.path.join(REF_DIR, REF_MODULE + ".so")
    srcs = [os.path.join(REFERENCE_OPS_DIR, f) for f in ("ops.cpp", "swap.cu", "ops.h")]
    if os.path.exists(so) and os.path.getmtime(so) >= max(os.path.getmtime(f) for f in srcs):
        return so
    os.makedirs(REF_DIR, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils import cpp_extension

    cpp_extension.load(
        name=REF_MODULE,
        sources=[os.path.join(REFERENCE_OPS_DIR, "ops.cpp"), os.path.join(REFERENCE_OPS_DIR, "swap.cu")],
        extra_include_paths=[REFERENCE_OPS_DIR],
        extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "-O2"],
        build_directory=REF_DIR,
        verbose=verbose,
        with_cuda=True,
    )
    # Drop intermediate build files; keep only the module.
    for f in os.listdir(REF_DIR):
        p = os.path.join(REF_DIR, f)
        if p != so and os.path.isfile(p) and not f.endswith(".so"):
            os.remove(p)
        elif os.path.isdir(p):
            shutil.rmtree(p)
    return so


if __name__ == "__main__":
    print(build_oracle_lib(force="--force" in sys.argv))
    print(build_reference_ops(verbose="-v" in sys.argv))
