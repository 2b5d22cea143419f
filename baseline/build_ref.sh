#!/usr/bin/env bash
# Build the reference implementation (Di-Chai/Centrifuge) for bench.py's reference arm.
#
#   baseline/build_ref.sh [reference source dir]     (default: $CFB_REFERENCE_SRC or /root/reference)
#
# The result is baseline/_ref: a copy of the reference source tree with its grad_filter
# extension built in place, exactly as the reference's own grad_filter/build.sh does it
# (python gen.py, then build_ext --inplace --define RESTORE_Q).  The source tree is copied
# because gen.py regenerates node_processing.cpp in place.  No reference source is edited.
# Two build-environment settings are needed with torch 2.11 on this image:
#   * CFLAGS="-include baseline/ref_compat.h": torch 2.11 added a fifth parameter to
#     Node::add_input_metadata, which the reference calls with four (node_processing.cpp:13);
#     the force-included header supplies the dtype argument.
#   * CXX=/usr/bin/g++: the default toolchain here links libstdc++ statically into extensions,
#     which leaves std::cout uninitialised inside them; the reference prints through std::cout.
#     The system g++ is the same GCC (13.3) that torch was built with and links libstdc++.so.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
SRC="${1:-${CFB_REFERENCE_SRC:-/root/reference}}"
OUT="$HERE/_ref"
if [ ! -f "$SRC/grad_filter/setup.py" ]; then
  echo "reference source not found at $SRC" >&2
  exit 2
fi
WORK="$(mktemp -d /tmp/cfb_ref_build.XXXXXX)"
cp -r "$SRC/." "$WORK/"
rm -rf "$WORK/.git"
chmod -R u+w "$WORK"
cd "$WORK/grad_filter"
python gen.py > "$WORK/gen.log" 2>&1
CXX=/usr/bin/g++ CC=/usr/bin/gcc CFLAGS="-include $HERE/ref_compat.h" \
  python setup.py build_ext --inplace --define RESTORE_Q > "$WORK/build.log" 2>&1 || {
    tail -30 "$WORK/build.log" >&2
    exit 1
  }
rm -rf "$WORK/grad_filter/build"
rm -rf "$OUT"
mv "$WORK" "$OUT"
echo "reference built into $OUT"
