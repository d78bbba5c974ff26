#!/usr/bin/env bash
# Regenerates tests/golden/golden.bin.gz and golden.json with the reference's own code
# (oracle/_ref/make_golden: make_golden.cpp compiled against the reference's reference.cpp and
# headers). Needs the reference tree: REF, else KVB_REF_DIR, else a `reference` directory beside
# this repository.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
make -C "$here/../../oracle" _ref/make_golden REF="${REF:-${KVB_REF_DIR:-$(cd "$here/../../.." && pwd)/reference}}"
"$here/../../oracle/_ref/make_golden" "$here/golden.bin" "$here/golden.json"
gzip -9 -n -f "$here/golden.bin"
