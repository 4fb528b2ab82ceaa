#!/usr/bin/env bash
# Test infrastructure only: builds the UNMODIFIED reference package
# (luisrodolfo10/diff_gabor_splatting v0.1.1, its Python API plus its CUDA
# extension `gabor_splatting._C`) for sm_100a into oracle/_ref/, so that GPU
# parity tests and the reference-extension timing script can run it on a B200
# (they import it as `gs_reference`, oracle/reference.py), and copies the
# reference's own test files into oracle/_ref_tests/ (oracle/fetch_ref_tests.sh).
#
# The reference source tree is read-only, so it is copied to a scratch directory
# and built there with its own setup.py (torch CUDAExtension, the flags it ships:
# -O3 -lineinfo) and TORCH_CUDA_ARCH_LIST=10.0a.  Nothing from the reference is
# committed: oracle/_ref/ is git-ignored and only travels with the working tree to
# the GPU box.
#
# usage: oracle/build_ref.sh [reference_dir]
#        (default: $GS_REFERENCE_DIR, else a checkout named `reference` beside this
#        repository)
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
src="${1:-${GS_REFERENCE_DIR:-$here/../../reference}}"
out="$here/_ref"
if [ ! -f "$src/setup.py" ]; then
    echo "reference source not found at $src; skipping" >&2
    exit 0
fi
bash "$here/fetch_ref_tests.sh" "$src"
if [ -f "$out/.built" ] && [ "$out/.built" -nt "$src/src/gabor_splatting/csrc/rasterize.cu" ]; then
    echo "reference already built in $out"
    exit 0
fi
scratch="$(mktemp -d "${TMPDIR:-/tmp}/gs_ref_build.XXXXXX")"
trap 'rm -rf "$scratch"' EXIT
cp -r "$src/." "$scratch/"
rm -rf "$out"
mkdir -p "$out"
TORCH_CUDA_ARCH_LIST="10.0a" MAX_JOBS="${MAX_JOBS:-4}" \
    python -m pip install --no-index --no-build-isolation --no-deps \
    --target "$out" "$scratch" >"$out/build.log" 2>&1
touch "$out/.built"
echo "reference built into $out"
