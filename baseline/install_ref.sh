#!/bin/bash
# Install the unmodified reference (ASarych/HTRC) into baseline/_ref for bench.py's reference legs.
#   bash baseline/install_ref.sh <reference checkout>
# The reference's own package (src/htrc_reference) is installed by pip from a temporary copy (its build writes
# into the source tree).  Its flat operator lives in h3/, which its pyproject does not package, so the h3
# directory is copied beside it unchanged.  baseline/_ref is git-ignored; it travels with the working tree.
set -euo pipefail
src=${1:?usage: install_ref.sh <reference checkout>}
here=$(cd "$(dirname "$0")" && pwd)
tmp=$(mktemp -d)
trap 'rm -rf "$tmp"' EXIT
cp -r "$src" "$tmp/ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$here/_ref" "$tmp/ref"
rm -rf "$here/_ref/h3"
cp -r "$src/h3" "$here/_ref/h3"
echo "installed into $here/_ref"
