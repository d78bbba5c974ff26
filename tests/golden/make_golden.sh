#!/usr/bin/env bash
# Regenerates tests/golden/golden.bin.gz and golden.json with the reference's own code
# (oracle/_ref/make_golden: make_golden.cpp compiled against the reference's reference.cpp and
# headers). Needs the reference tree (REF, default /root/reference).
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
make -C "$here/../../oracle" _ref/make_golden REF="${REF:-/root/reference}"
"$here/../../oracle/_ref/make_golden" "$here/golden.bin" "$here/golden.json"
gzip -9 -n -f "$here/golden.bin"
