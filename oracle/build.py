"""Build recipe for the oracle's native parts -- TEST INFRASTRUCTURE ONLY.

  oracle/liboracle_bsr.so   the plain-C restatement (bsr_oracle.c), built with gcc everywhere
  oracle/_ref/libbsr_ref.so the reference's own cpu_bsr (build_ref.sh), built only when the location of a
                            reference checkout is given (argument `ref_root` or REF_ROOT) and holds the source
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle_bsr.so")
REF_LIB = os.path.join(HERE, "_ref", "libbsr_ref.so")


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "bsr_oracle.c")
    if force or not os.path.exists(ORACLE_LIB) or os.path.getmtime(src) > os.path.getmtime(ORACLE_LIB):
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-shared", "-fPIC", src, "-o", ORACLE_LIB], check=True)
    return ORACLE_LIB


def build_ref(force: bool = False, ref_root: str | None = None) -> str | None:
    """Builds oracle/_ref from the reference checkout at `ref_root` (default: $REF_ROOT); without one, returns the
    library built earlier, if any."""
    ref_root = ref_root or os.environ.get("REF_ROOT")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "BlackwellSparseK", "src")):
        return REF_LIB if os.path.exists(REF_LIB) else None
    if force or not os.path.exists(REF_LIB):
        subprocess.run(["sh", os.path.join(HERE, "build_ref.sh")], check=True, stdout=subprocess.DEVNULL,
                       env={**os.environ, "REF_ROOT": ref_root})
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force=True), build_ref(force=True))
