#!/bin/sh
# Builds the test oracle (CPU restatement of the reference index algorithms).
# -ffp-contract=off keeps every fmaf/mul/add exactly as written.
set -e
here="$(cd "$(dirname "$0")" && pwd)"
gcc -O2 -ffp-contract=off -fPIC -shared -std=c11 -o "$here/libmi_oracle.so" "$here/mi_oracle.c" -lm
