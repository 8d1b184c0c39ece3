#!/bin/bash
# Installs the reference checkout's src/ modules, unmodified, under baseline/_ref
# (git-ignored; it travels to the GPU box with the repository), for bench.py's
# same-box comparison with the reference's Triton grouped GEMM.  The checkout has
# neither setup.py nor pyproject.toml, so a copy under a temporary directory gets a
# packaging shim that lists the modules; the module files themselves are installed
# byte for byte, which the last step checks.
# usage: baseline/install_reference.sh <reference checkout>
set -euo pipefail
SRC=${1:?usage: baseline/install_reference.sh <reference checkout>}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT
mkdir -p "$TMP/src"
cp "$SRC"/src/*.py "$TMP/src/"
MODULES=$(cd "$TMP/src" && ls *.py | sed 's/\.py$//' | awk '{printf "\"%s\", ", $0}')
cat > "$TMP/setup.py" <<PY
from setuptools import setup
setup(name="moe_overlap_reference", version="0", package_dir={"": "src"},
      py_modules=[$MODULES])
PY
python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
    --target "$HERE/_ref" --no-deps --upgrade "$TMP"
for f in "$SRC"/src/*.py; do cmp "$f" "$HERE/_ref/$(basename "$f")"; done
echo "installed $(ls "$SRC"/src/*.py | wc -l) reference modules under $HERE/_ref, unmodified"
