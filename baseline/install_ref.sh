#!/bin/sh
# Installs the unmodified Tokquay reference into baseline/_ref (git-ignored; it travels
# with the repository snapshot to GPU boxes, where bench.py's reference arm and the
# reference-engine tests import it).
#
# The reference is a uv project that runs from its source root (pytest's
# pythonpath = ["."]); its pyproject has no package list, so pip cannot build it
# as is: setuptools stops with "Multiple top-level packages discovered in a
# flat-layout: ['bench', 'tokquay', 'Documentation']".  This script copies the
# two Python packages, byte for byte, into a scratch build directory under /tmp,
# adds a two-line setup.py naming them, and installs that with pip, offline.
# --no-deps: the image's fastapi / numpy / transformers are older than the
# reference's floor pins and matplotlib is absent, none of which the paged path
# or the engine imports; --ignore-requires-python: the reference asks for
# Python >= 3.13 and runs unchanged on this image's 3.12.
#
# Usage: baseline/install_ref.sh <path to the reference checkout>
set -eu
src=${1:?usage: $0 <reference checkout>}
here=$(cd "$(dirname "$0")" && pwd)
build=$(mktemp -d /tmp/tokquay_ref_build.XXXXXX)
cp -r "$src/tokquay" "$src/bench" "$build/"
find "$build" -name __pycache__ -prune -exec rm -rf {} +
cat > "$build/setup.py" <<'PY'
from setuptools import setup
setup(name="tokquay", version="0.1.0", packages=["tokquay", "bench"])
PY
rm -rf "$here/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --ignore-requires-python \
    --find-links /opt/wheelhouse --target "$here/_ref" "$build"
rm -rf "$build"
# record what was installed: file list with checksums of the reference's sources
(cd "$src" && find tokquay bench -name '*.py' | sort | xargs sha256sum) > "$here/_ref/SOURCES.sha256"
