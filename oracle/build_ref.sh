#!/usr/bin/env bash
# Builds the reference's own CPU solver from its sources, in place, into
# oracle/_ref/.  It is test infrastructure only: the parity tests use it to pin
# the C++ restatement in oracle/, and bench.py's reference arm times it.
#
#   _duck_reference<EXT_SUFFIX>  src/cuda/cpu_bindings.cpp + src/solver.cpp
#       (CpuBatch32/CpuBatch64, convex_query32/64; the same kernel.cuh the
#        reference compiles for CUDA, built for the host)
#   duck_sim                     src/main.cpp + src/solver.cpp (legacy FP64)
#
# The direct g++ line is used instead of the reference's CMake build: the
# CMake/pybind11 build of this module segfaulted in its constructor when numpy
# was imported first, the direct build does not.  Flags follow the reference's
# CMakeLists.txt (-O3, -ffp-contract=off).
#
# DUCK_REFERENCE names the reference checkout; without it nothing is built.
set -euo pipefail
REF=${DUCK_REFERENCE:-}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
if [ -z "$REF" ] || [ ! -f "$REF/src/cuda/kernel.cuh" ]; then
  echo "reference sources not found (DUCK_REFERENCE='$REF'); skipping oracle/_ref" >&2
  exit 0
fi
mkdir -p "$OUT"
PY=${PYTHON:-python3}
EXT=$($PY -c "import sysconfig;print(sysconfig.get_config_var('EXT_SUFFIX'))")
PYINC=$($PY -c "import sysconfig;print(sysconfig.get_paths()['include'])")
PBINC=$($PY -c "import pybind11;print(pybind11.get_include())")
/usr/bin/g++ -O3 -DNDEBUG -std=c++17 -fPIC -fvisibility=hidden -shared -Wno-narrowing \
  -ffp-contract=off -I"$REF/include" -isystem "$PYINC" -isystem "$PBINC" \
  "$REF/src/cuda/cpu_bindings.cpp" "$REF/src/solver.cpp" \
  -o "$OUT/_duck_reference$EXT" -lpthread
/usr/bin/g++ -O3 -DNDEBUG -std=c++17 -ffp-contract=off -I"$REF/include" \
  "$REF/src/main.cpp" "$REF/src/solver.cpp" -o "$OUT/duck_sim"
echo "built $OUT/_duck_reference$EXT and $OUT/duck_sim"
