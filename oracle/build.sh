#!/usr/bin/env bash
# Builds the CPU checker (test infrastructure only):
#   oracle/liboracle.so            the C restatement (oracle.c, shifts.cpp), always
#   oracle/_ref/libstems_ref.so    the reference's own stft.h / vr_dsp.h behind ref_shim.cpp,
#   oracle/_ref/dsp_test           the reference's own known-answer tests, compiled from its
#   oracle/_ref/vr_dsp_test        sources where they lie,
# the last three only when the reference sources are present (REF_SRC or ../reference).
# Flags follow the reference's Release build (CMakeLists.txt: C++17, CMAKE_BUILD_TYPE Release).
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF_ROOT="${REF_ROOT:-$HERE/../../reference}"
REF_SRC="${REF_SRC:-$REF_ROOT/src}"

OBJ="$(mktemp -d)"
trap 'rm -rf "$OBJ"' EXIT
gcc -O2 -std=c11 -fPIC -Wall -Wno-unused-result -c "$HERE/oracle.c" -o "$OBJ/oracle.o"
g++ -O2 -std=c++17 -fPIC -Wall -c "$HERE/shifts.cpp" -o "$OBJ/shifts.o"
g++ -shared "$OBJ/oracle.o" "$OBJ/shifts.o" -o "$HERE/liboracle.so" -lm -lpthread -ldl

if [ -f "$REF_SRC/stft.h" ] && [ -f "$REF_SRC/vr_dsp.h" ]; then
    mkdir -p "$HERE/_ref"
    g++ -O3 -DNDEBUG -std=c++17 -fPIC -shared -I"$REF_SRC" "$HERE/ref_shim.cpp" -o "$HERE/_ref/libstems_ref.so"
    if [ -f "$REF_ROOT/tests/dsp_test.cpp" ]; then
        g++ -O3 -DNDEBUG -std=c++17 -I"$REF_SRC" "$REF_ROOT/tests/dsp_test.cpp" -o "$HERE/_ref/dsp_test"
    fi
    if [ -f "$REF_ROOT/tests/vr_dsp_test.cpp" ]; then
        g++ -O3 -DNDEBUG -std=c++17 -I"$REF_SRC" "$REF_ROOT/tests/vr_dsp_test.cpp" -o "$HERE/_ref/vr_dsp_test"
    fi
    echo "oracle: built restatement and reference ($REF_SRC)"
else
    echo "oracle: built restatement (reference sources absent; oracle/_ref left as is)"
fi
