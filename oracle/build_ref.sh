#!/usr/bin/env bash
# Build the reference's shipped C-ABI library (one CUDA source file, cuBLASLt
# from the CUDA toolkit) for sm_100a into oracle/_ref/, as a cross-check of
# the W8A8 path in the GPU tests.  Test infrastructure only; outputs stay
# under oracle/_ref/ (git-ignored, carried to the GPU box with the tree).
#
#   bash oracle/build_ref.sh [REFERENCE_ROOT]
#
# REFERENCE_ROOT: the reference checkout (argument, else $MOSYNE_REFERENCE_ROOT,
# else a directory named "reference" beside this repository).
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${1:-${MOSYNE_REFERENCE_ROOT:-$HERE/../../reference}}
SRC="$REF/packages/mosyne_bposit/src/mosyne_bposit/_cuda/libmosyne_bposit.cu"
if [ ! -f "$SRC" ]; then echo "reference sources not present; nothing to build"; exit 0; fi
mkdir -p "$HERE/_ref"
nvcc -O3 -std=c++17 -shared -Xcompiler -fPIC \
     -gencode arch=compute_100a,code=sm_100a \
     "$SRC" -o "$HERE/_ref/libmosyne_bposit_ref.so" -lcublasLt -lcudart
echo "$HERE/_ref/libmosyne_bposit_ref.so"
