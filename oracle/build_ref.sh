#!/bin/sh
# Compiles the reference's CPU BSR checker (cpu_bsr, BlackwellSparseK/src/bsr_reference.cu) from its
# source in the reference checkout into oracle/_ref/libbsr_ref.so -- TEST INFRASTRUCTURE ONLY.
# REF_ROOT names the directory that holds the reference checkout (BlackwellSparseK/ inside it); required.
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
[ -n "$REF_ROOT" ] || { echo "set REF_ROOT to the reference checkout" >&2; exit 2; }
SRC="$REF_ROOT/BlackwellSparseK/src/bsr_reference.cu"
[ -f "$SRC" ] || { echo "reference source not found: $SRC" >&2; exit 2; }
mkdir -p "$HERE/_ref"
CUDA_HOME=${CUDA_HOME:-/usr/local/cuda}
"$CUDA_HOME/bin/nvcc" -O2 -std=c++17 -shared -Xcompiler -fPIC -Xcompiler -ffp-contract=off \
  -DBSK_REF_SRC="\"$SRC\"" "$HERE/ref_wrap.cu" -lcublas -Xlinker -rpath="$CUDA_HOME/lib64" \
  -o "$HERE/_ref/libbsr_ref.so"
echo "built $HERE/_ref/libbsr_ref.so"
