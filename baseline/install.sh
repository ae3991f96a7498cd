#!/bin/sh
# Install the reference (omin-Kwon/nested_ssm) into baseline/_ref for bench.py's same-box run
# of the reference's own GPU decode arms (scale/bench_v4_decode.py run_point).
#
#   sh baseline/install.sh <checkout of omin-Kwon/nested_ssm>
#
# The reference is a research tree without packaging metadata, so `pip install <tree>` has
# nothing to build.  This copies its scale/*.py modules, unmodified, into a temporary
# directory, adds a minimal pyproject.toml that names them as top-level modules, and installs
# that with pip (no index, no dependencies: torch, triton and fla come from the environment).
set -eu
REF=${1:?usage: sh baseline/install.sh <checkout of omin-Kwon/nested_ssm>}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
trap 'rm -rf "$TMP"' EXIT
cp "$REF"/scale/*.py "$TMP"/
MODS=$(cd "$TMP" && ls *.py | sed 's/\.py$//' | awk '{printf "%s\"%s\"", (NR>1?", ":""), $0}')
cat > "$TMP/pyproject.toml" <<TOML
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "nested-ssm-reference"
version = "0.0.0"

[tool.setuptools]
py-modules = [$MODS]
TOML
python -m pip install --no-index --no-build-isolation --no-deps --target "$HERE/_ref" "$TMP"
