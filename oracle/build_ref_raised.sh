#!/usr/bin/env bash
# Builds the reference's own CPU solver (src/cuda/cpu_bindings.cpp +
# src/solver.cpp, the same kernel.cuh as its CUDA path) with the body-collision
# pair capacity raised from 32 to 128, into oracle/_ref/raised/ as
# _duck_reference_raised<EXT_SUFFIX>.  Test infrastructure only: it pins this
# repository's raised-limit oracle (OracleBatch(max_pairs=128)) to the
# reference's arithmetic on models with more than 32 pairs, which the
# unmodified reference rejects.
#
# The reference sources are copied to a temporary directory outside the
# repository and four constants are changed there (a declared deviation):
#   src/solver.cpp      loader: pair count limit 32 -> 128
#   src/cuda/model.hpp  convert: collisionPairs.size() <= 32 -> <= 128
#   src/cuda/kernel.cuh Model::pairs List<CollisionPair, 32> -> 128
#   src/cuda/cpu_bindings.cpp module name _duck_reference -> _duck_reference_raised
# The generic state's contact capacity (160) already covers 91 pairs plus four
# contacts per ground shape (151 for the 15-shape biped).  Flags as
# oracle/build_ref.sh.  DUCK_REFERENCE names the reference checkout.
set -euo pipefail
REF=${DUCK_REFERENCE:-}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref/raised"
if [ -z "$REF" ] || [ ! -f "$REF/src/cuda/kernel.cuh" ]; then
  echo "reference sources not found (DUCK_REFERENCE='$REF'); skipping oracle/_ref/raised" >&2
  exit 0
fi
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT
cp -r "$REF/src" "$REF/include" "$TMP/"
patch_line() {  # file, old, new: exactly one occurrence must change
  local file=$1 old=$2 new=$3
  [ "$(grep -cF -- "$old" "$file")" = 1 ] || { echo "expected one '$old' in $file" >&2; exit 1; }
  python3 - "$file" "$old" "$new" <<'PY'
import sys
path, old, new = sys.argv[1:]
text = open(path).read()
open(path, "w").write(text.replace(old, new))
PY
}
patch_line "$TMP/src/solver.cpp" "count < 0 || count > 32)" "count < 0 || count > 128)"
patch_line "$TMP/src/cuda/model.hpp" "original.collisionPairs.size() <= 32," "original.collisionPairs.size() <= 128,"
patch_line "$TMP/src/cuda/kernel.cuh" "List<CollisionPair, 32> pairs;" "List<CollisionPair, 128> pairs;"
patch_line "$TMP/src/cuda/cpu_bindings.cpp" "PYBIND11_MODULE(_duck_reference," "PYBIND11_MODULE(_duck_reference_raised,"
mkdir -p "$OUT"
PY=${PYTHON:-python3}
EXT=$($PY -c "import sysconfig;print(sysconfig.get_config_var('EXT_SUFFIX'))")
PYINC=$($PY -c "import sysconfig;print(sysconfig.get_paths()['include'])")
PBINC=$($PY -c "import pybind11;print(pybind11.get_include())")
/usr/bin/g++ -O3 -DNDEBUG -std=c++17 -fPIC -fvisibility=hidden -shared -Wno-narrowing \
  -ffp-contract=off -I"$TMP/include" -isystem "$PYINC" -isystem "$PBINC" \
  "$TMP/src/cuda/cpu_bindings.cpp" "$TMP/src/solver.cpp" \
  -o "$OUT/_duck_reference_raised$EXT" -lpthread
echo "built $OUT/_duck_reference_raised$EXT"
