#!/usr/bin/env bash
# Test infrastructure only: copies the reference's own rendering and spherical-
# harmonics test files (tests/test_rendering.py, tests/test_spherical_harmonics.py of
# luisrodolfo10/diff_gabor_splatting v0.1.1), unmodified, into oracle/_ref_tests/.
# tests/test_reference_suite_gpu.py runs them there against this repository's
# `gabor_splatting` drop-in package.  oracle/_ref_tests/ is git-ignored (the files are
# the reference's, not this project's) and travels with the working tree to the GPU
# box.  test_upstream.py is not copied: it needs the pinned upstream rasterizers,
# which are not installed.
#
# usage: oracle/fetch_ref_tests.sh [reference_dir]
#        (default: $GS_REFERENCE_DIR, else a checkout named `reference` beside this
#        repository)
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
src="${1:-${GS_REFERENCE_DIR:-$here/../../reference}}"
out="$here/_ref_tests"
if [ ! -f "$src/tests/test_rendering.py" ]; then
    echo "reference tests not found under $src; skipping" >&2
    exit 0
fi
mkdir -p "$out"
for name in test_rendering.py test_spherical_harmonics.py; do
    cp "$src/tests/$name" "$out/$name"
done
echo "reference tests copied into $out"
