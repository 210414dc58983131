#!/usr/bin/env bash
# TEST INFRASTRUCTURE (oracle). Compiles the reference's own CPU kernels from its patch into oracle/_ref/:
#   oracle/_ref/srv-kernels.inc   the new file ggml/src/ggml-cpu/srv-kernels.inc of patch/srhpm.patch (777 lines)
#   oracle/_ref/fa-gqa.inc        the FA-GQA block added to ggml/src/ggml-cpu/ops.cpp (patch/srhpm.patch:539-824)
#   oracle/_ref/libsrv_ref_avx2.so  driver + kernels, AVX2 build (no VNNI: vpmaddwd + vpaddd path)
#   oracle/_ref/libsrv_ref_vnni.so  same with AVX-VNNI (vpdpwssd path), built when the compiler accepts -mavxvnni
# The reference's build system (cmake over the llama.cpp tree) is not used: the tree is not in the container.
# Only the patch's own added lines are compiled, against the stand-ins in oracle/ref_shim.h and
# oracle/ggml_restated.h. Usage: oracle/build_ref.sh <path-to-reference> (or set SRHPM_REFERENCE)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${SRHPM_REFERENCE:-}}"
if [ -z "$REF" ]; then
    echo "build_ref: give the reference checkout as the argument or in SRHPM_REFERENCE" >&2
    exit 2
fi
PATCH="$REF/patch/srhpm.patch"
OUT="$HERE/_ref"
if [ ! -f "$PATCH" ]; then
    echo "build_ref: no reference patch at $PATCH" >&2
    exit 2
fi
mkdir -p "$OUT"

# srv-kernels.inc: every line of the new-file hunk, '+' stripped
awk '
    /^diff --git a\/ggml\/src\/ggml-cpu\/srv-kernels.inc / { infile = 1; next }
    infile && /^diff --git / { exit }
    infile && /^@@ / { body = 1; next }
    infile && body { sub(/^\+/, ""); print }
' "$PATCH" > "$OUT/srv-kernels.inc"
n=$(wc -l < "$OUT/srv-kernels.inc")
if [ "$n" -ne 777 ]; then
    echo "build_ref: srv-kernels.inc has $n lines, expected 777 (patch changed?)" >&2
    exit 3
fi

# FA-GQA: from its opening comment to the closing brace of ggml_compute_forward_flash_attn_ext_gqa_small
awk '
    /^\+\/\/ SR-HPM \(SRHPM_FA_GQA=1\)/ { on = 1 }
    on && /^ static void ggml_compute_forward_flash_attn_ext_f16\(/ { exit }
    on { sub(/^\+/, ""); print }
' "$PATCH" > "$OUT/fa-gqa.inc"
n=$(wc -l < "$OUT/fa-gqa.inc")
if [ "$n" -ne 287 ]; then
    echo "build_ref: fa-gqa.inc has $n lines, expected 287 (patch changed?)" >&2
    exit 3
fi

CXXFLAGS="-O3 -std=c++17 -fPIC -shared -Wno-unused-function -Wno-ignored-attributes -I$HERE -I$OUT"
g++ $CXXFLAGS -mavx2 -mfma -mf16c "$HERE/srv_ref_driver.cpp" -o "$OUT/libsrv_ref_avx2.so" -lpthread
if echo 'int main(){}' | g++ -mavxvnni -x c++ - -o /dev/null 2>/dev/null; then
    g++ $CXXFLAGS -mavx2 -mfma -mf16c -mavxvnni "$HERE/srv_ref_driver.cpp" -o "$OUT/libsrv_ref_vnni.so" -lpthread
fi
echo "build_ref: ok ($OUT)"
