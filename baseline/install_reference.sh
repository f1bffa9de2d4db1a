#!/bin/sh
# Install the unmodified LinkQ2 reference into baseline/_ref (git-ignored) and place its
# own test files beside it, so that baseline/reference_gpu.py can run the reference's GPU
# path and the reference's tests where no checkout of the reference exists.
#
#   sh baseline/install_reference.sh /path/to/LinkQ2
#
# The install builds a wheel, which writes into the source tree, so a read-only checkout
# is copied to a scratch directory first.  Dependencies are not resolved (--no-deps): the
# reference pins torch 2.7.1 / triton 3.3.1 / transformers 4.57.6, the image has newer ones.
set -e
SRC=${1:?usage: install_reference.sh /path/to/LinkQ2}
HERE=$(cd "$(dirname "$0")" && pwd)
TMP=$(mktemp -d)
cp -r "$SRC" "$TMP/src"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
    --target "$HERE/_ref" --upgrade "$TMP/src"
rm -rf "$HERE/_ref/reference_tests"
cp -r "$SRC/tests" "$HERE/_ref/reference_tests"
cp "$SRC/pytest.ini" "$HERE/_ref/pytest.ini"
rm -rf "$TMP"
echo "installed into $HERE/_ref"
