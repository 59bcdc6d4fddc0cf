#!/bin/bash
# Writes compat_suite_b200.json and compat_suite_b200_trace.jsonl: the compat bench's suite
# scenario (four padded 37 x 19 x 67 shapes with the ordinary-cuBLAS baseline, an
# out-of-core 4096 x 3072 x 2048 GEMM through a 64 MiB cache, the rejection set) run on a
# B200.  tests/test_report_contracts_cpu.py checks them with the reference's compat
# contract.  Usage: make_compat_suite_b200.sh [output directory, default: this directory]
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
out="${1:-$here}"
mkdir -p "$out"
cd "$here/../.."
python -m xvram_b200.compat_bench --scenario suite --m 4096 --n 3072 --k 2048 \
    --padding 3 --offset 5 --passes 2 --beta 1 --cache-target-mib 64 --chunk-mib 2 \
    --report "$out/compat_suite_b200.json" --trace "$out/compat_suite_b200_trace.jsonl"
