#!/usr/bin/env bash
# Installs the unmodified reference (jyotilakra92/nifre) into baseline/_ref so
# that bench.py can time the reference's own CPU attention path on the GPU box
# (baseline/_ref is git-ignored and travels with the repository snapshot).
# The reference ships no packaging metadata, so the recipe copies it to /tmp,
# adds a pyproject.toml that only declares the src/ layout, and installs that
# copy; no reference source file is changed.
set -euo pipefail
REF=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d /tmp/nifre_ref.XXXXXX)
mkdir -p "$TMP/src"
cp -r "$REF/src/inference" "$REF/src/sampler.py" "$TMP/src/"
cat > "$TMP/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "nifre-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
where = ["src"]
include = ["inference*"]

[tool.setuptools]
py-modules = ["sampler"]
TOML
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" --upgrade "$TMP"
rm -rf "$TMP"
