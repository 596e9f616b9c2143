#!/usr/bin/env bash
# Install the unmodified reference (kagami4243/extend-nano-vLLM 0.3.0) into
# baseline/_ref, offline, for the GPU tests that run its Triton path
# (tests/test_gpu_reference_triton.py).  The source tree is copied to a
# temporary directory first because the build writes into the tree.
#   REFERENCE_ROOT=/path/to/extend-nano-vLLM baseline/install_reference.sh
set -euo pipefail
: "${REFERENCE_ROOT:?set REFERENCE_ROOT to the extend-nano-vLLM source tree}"
here="$(cd "$(dirname "$0")" && pwd)"
tmp="$(mktemp -d)"
trap 'rm -rf "$tmp"' EXIT
cp -r "$REFERENCE_ROOT" "$tmp/src"
python -m pip install --no-index --no-build-isolation --no-deps \
    --find-links /opt/wheelhouse --target "$here/_ref" "$tmp/src"
