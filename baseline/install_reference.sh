#!/bin/sh
# Installs the reference (inin-zou/kernelgen-challenge, track-01) for the
# comparison legs of bench.py: its unmodified Python files copied into
# baseline/_ref/track-01 (git-ignored).  The reference is a pure-Python
# repository with no setup.py or pyproject.toml, so `pip install --target`
# refuses it ("not installable"); a plain copy is the install.
#   usage: sh baseline/install_reference.sh <path of the reference checkout>
set -e
src="${1:?path of the reference checkout}"
here="$(cd "$(dirname "$0")" && pwd)"
mkdir -p "$here/_ref/track-01/reference"
cp "$src/track-01/submission.py" "$src/track-01/workloads.py" "$here/_ref/track-01/"
cp "$src/track-01/reference/__init__.py" "$src/track-01/reference/reference.py" \
   "$here/_ref/track-01/reference/"
echo "installed into $here/_ref/track-01"
