#!/usr/bin/env bash
# Compiles the reference's own C oracles straight out of the Go test files
# where they lie (tensor/oracle_q4_k_test.go, tensor/oracle_q6_k_test.go,
# tensor/oracle_c_test.go: the C source is a Go raw-string constant).  The
# source is piped to gcc on stdin, so nothing of it is written into this
# repository; only the binaries land in oracle/_ref/ (git-ignored).
# Flags follow the reference tests (oracle_q4_k_test.go:135, oracle_c_test.go:101).
# The reference tree: the first argument, else $C2S_REFERENCE, else a
# directory named "reference" beside this repository.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${C2S_REFERENCE:-$HERE/../../reference}}"
OUT="$HERE/_ref"
if [ ! -d "$REF/tensor" ]; then
  echo "reference tree not found at $REF; skipping _ref build" >&2
  exit 0
fi
mkdir -p "$OUT"
extract() {  # $1 = file, $2 = Go constant name
  awk -v name="$2" '
    $0 ~ "^const " name " = `" { on = 1; next }
    on && /^`/ { exit }
    on { print }' "$1"
}
extract "$REF/tensor/oracle_q4_k_test.go" cQ4_KSource | gcc -O2 -std=c99 -pedantic -Wall -Werror -x c - -lm -o "$OUT/q4_k_dequant"
extract "$REF/tensor/oracle_q6_k_test.go" cQ6_KSource | gcc -O2 -std=c99 -pedantic -Wall -Werror -x c - -lm -o "$OUT/q6_k_dequant"
extract "$REF/tensor/oracle_c_test.go"   cQ5_0Source | gcc -O2 -x c - -lm -o "$OUT/q5_0_dequant"
echo "built: $(ls "$OUT" | tr '\n' ' ')"
