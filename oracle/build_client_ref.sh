#!/bin/sh
# Builds oracle/_ref/bfp_client_ref: the reference client's own decode_tokens
# and fix_mojibake (compiled from the reference checkout, where its sources
# lie) behind the small stdin driver in client_ref_main.cpp.  Test
# infrastructure only: it makes the client fixtures and checks the Python
# port against them.
#
#   oracle/build_client_ref.sh [reference checkout, default ../reference]
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${1:-${BFP200_REFERENCE:-$HERE/../../reference}}
SRC="$REF/rtl/vc707/host/bfp_client.cpp"
if [ ! -f "$SRC" ]; then
  echo "build_client_ref: $SRC not found (reference checkout absent)" >&2
  exit 3
fi
mkdir -p "$HERE/_ref"
g++ -std=c++17 -O1 -w -Dmain=bfp_client_main "-DBFP_CLIENT_CPP=\"$SRC\"" \
    -o "$HERE/_ref/bfp_client_ref" "$HERE/client_ref_main.cpp" -lpthread
echo "built $HERE/_ref/bfp_client_ref"
