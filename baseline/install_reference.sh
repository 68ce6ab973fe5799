#!/bin/sh
# Installs the reference's `foreswe_bench` package (its Triton v1/v2 geo-attention kernels and the eager operator)
# into baseline/_ref, offline, for the on-GPU Triton v2 timing in `bench.py --workload configs`.
#
# The reference's pyproject.toml names no packages, and setuptools' flat-layout discovery refuses its tree (several
# top-level packages), so the recipe copies pyproject.toml and foreswe_bench/ to a scratch directory, lists the one
# package explicitly and installs from there (the reference checkout is read-only).
#
#   sh baseline/install_reference.sh <path of the reference checkout>
set -eu
REF="${1:?usage: sh baseline/install_reference.sh <path of the reference checkout>}"
HERE="$(cd "$(dirname "$0")" && pwd)"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp "$REF/pyproject.toml" "$TMP/"
cp -r "$REF/foreswe_bench" "$TMP/"
cat >> "$TMP/pyproject.toml" << 'EOT'

[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[tool.setuptools]
packages = ["foreswe_bench"]
EOT
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" "$TMP"
