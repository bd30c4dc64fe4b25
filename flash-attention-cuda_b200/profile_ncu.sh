#!/bin/bash
# ncu capture of the two kernels on their benchmark workloads, then a markdown
# summary (flashattn_cuda.ncu_extract). Run on a B200 from the repository root:
#
#   bash flash-attention-cuda_b200/profile_ncu.sh [OUT_DIR]
#
# Each workload first runs once without ncu (a failing program is never
# profiled); one launch per kernel is captured after two warm-up launches,
# always with --clock-control none so the GPU's clocks are left untouched.
set -euo pipefail
OUT=${1:-ncu_out}
PKG=flash-attention-cuda_b200
NCU=${NCU:-ncu}
mkdir -p "$OUT"
for spec in prefill_c3:prefill_kernel decode_c4:decode_kernel; do
  case_name=${spec%%:*}; kernel=${spec##*:}
  python "$PKG/profile_workload.py" --case "$case_name" > "$OUT/$case_name.plain.log" 2>&1
  "$NCU" --set full --clock-control none -k "regex:$kernel" -s 2 -c 1 \
      -o "$OUT/$case_name" -f python "$PKG/profile_workload.py" --case "$case_name" \
      > "$OUT/$case_name.ncu.log" 2>&1
  "$NCU" -i "$OUT/$case_name.ncu-rep" --page raw --csv > "$OUT/$case_name.csv"
done
(cd "$PKG" && python -m flashattn_cuda.ncu_extract --prefill "../$OUT/prefill_c3.csv" \
    --decode "../$OUT/decode_c4.csv" --out "../$OUT/ncu_summary.md")
echo "wrote $OUT/ncu_summary.md"
