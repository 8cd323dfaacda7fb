#!/bin/sh
# Installs the unmodified reference (Theophite/Concord) under baseline/_ref so
# that it travels to the GPU box.  The reference ships no packaging metadata,
# so the sources are copied to /tmp (the source tree is read-only) and a
# minimal pyproject naming its two importable parts is added beside them:
#   concord                       (concord/packed_b.py: the Triton kernels)
#   experiments.cpu_dynamics      (concord_ref.py: the real-valued CPU rule)
# Nothing in the copied sources is edited.
set -e
SRC=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d /tmp/concord_ref_src.XXXXXX)
cp -r "$SRC/concord" "$SRC/experiments" "$TMP/"
touch "$TMP/experiments/__init__.py" "$TMP/experiments/cpu_dynamics/__init__.py"
cat > "$TMP/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"
[project]
name = "concord-reference"
version = "0.0.0"
[tool.setuptools]
packages = ["concord", "experiments", "experiments.cpu_dynamics"]
TOML
python -m pip install --no-index --no-build-isolation --no-deps \
    --find-links /opt/wheelhouse --target "$HERE/_ref" "$TMP"
