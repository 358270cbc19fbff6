"""CPU oracle for the batmobile hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() (as the checker) and bench.py's CPU
baseline leg may import this package.  The product never does, and has no CPU
fallback through it.  Build the compiled pieces with `make -C oracle`.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(ref=None):
    """Compile oracle/_build (always) and oracle/_ref (when `ref`, or the
    BATMOBILE_REF environment variable, names an existing reference checkout)."""
    ref = ref or os.environ.get("BATMOBILE_REF", "")
    subprocess.run(["make", "-s", "-C", HERE, "REF=" + ref], check=True)
    if ref and os.path.isdir(os.path.join(ref, "src")):
        from . import ref_cuda   # the reference's CUDA kernels for sm_100a (comparison arm)
        ref_cuda.build(ref)
