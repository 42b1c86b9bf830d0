#!/bin/sh
# Installs the unmodified reference sources into baseline/_ref for bench.py's
# reference arm.
#
# The reference ships no build system (no setup.py or pyproject.toml), so a pip
# install of its tree fails with "Neither 'setup.py' nor 'pyproject.toml'
# found". This script copies the tree to a temporary directory, adds a
# packaging-only pyproject.toml that declares its two modules
# (src/numa_all_reduce.py, src/numa_utils.py), and pip-installs that copy
# offline. No reference source file is changed.
#
# usage: sh baseline/install_ref.sh <reference-source-dir>
set -eu
src="$1"
here="$(cd "$(dirname "$0")" && pwd)"
tmp="$(mktemp -d /tmp/nab_ref.XXXXXX)"
cp -r "$src/." "$tmp/"
cat > "$tmp/pyproject.toml" <<'TOML'
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "numa-allreduce-reference"
version = "0.0.0"

[tool.setuptools]
package-dir = {"" = "src"}
py-modules = ["numa_all_reduce", "numa_utils"]
TOML
python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
    --target "$here/_ref" --no-deps "$tmp"
rm -rf "$tmp"
