#!/bin/sh
# Installs the reference package into baseline/_ref (git-ignored; it travels
# to the GPU box with the rest of the tree). The GPU comparator in
# baseline/triton_comparator.py runs the reference's own Triton kernels from
# there; nothing else reads it.
#
#   sh baseline/install_ref.sh /path/to/reference-checkout
#
# The reference checkout is a bare package directory (elastikernel/) with no
# setup.py or pyproject.toml, so pip rejects it ("not installable"); the
# package directory is then placed under baseline/_ref unmodified.
set -eu
REF=${1:?usage: install_ref.sh REFERENCE_ROOT}
HERE=$(cd "$(dirname "$0")" && pwd)
if python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --target "$HERE/_ref" "$REF"; then
  exit 0
fi
echo "pip could not install $REF; placing its package directory under baseline/_ref" >&2
mkdir -p "$HERE/_ref"
rm -rf "$HERE/_ref/elastikernel"
cp -r "$REF/elastikernel" "$HERE/_ref/elastikernel"
find "$HERE/_ref/elastikernel" -name __pycache__ -type d -prune -exec rm -rf {} +
