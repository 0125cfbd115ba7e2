#!/bin/bash
# Runs the reference's own harness, tools/bench.py (and, with "ncu", tools/ncu_profile.py), with
# this repository's plugin modules in its kernel slot -- TEST INFRASTRUCTURE, the drop-in check.
#
#   bash oracle/run_reference_harness.sh [REFERENCE_CHECKOUT] [OUT_DIR] [ncu]
#
# REFERENCE_CHECKOUT (default /root/reference) is copied to a scratch directory; its kernel.py
# becomes the two-line shim of INTEGRATION.md for each module in turn and tools/bench.py runs
# unmodified.  The one change in the copy: the reference builds its scalar GDN checker kernel for
# sm_89 SASS only, which a B200 cannot run, so that build flag is retargeted to sm_100a.
set -u
HERE=$(cd "$(dirname "$0")/.." && pwd)
REF=${1:-/root/reference}
OUT=${2:-$HERE/gpurun_out}
SCRATCH=$(mktemp -d /tmp/refharness.XXXXXX)
mkdir -p "$OUT"
cp -r "$REF"/. "$SCRATCH"/
cd "$SCRATCH"
sed -i 's/compute_89,code=sm_89/compute_100a,code=sm_100a/' kernels/*.py kernels_optimized/*.py
export PYTHONPATH=$HERE
rc=0
for mod in qwen35moe_gdn_prefill flash_attention_2; do
  printf '# kernel slot: %s on the sm_100a kernels\nfrom kernel_opt_agent_b200.%s import KERNEL_TYPE, kernel_fn, get_inputs, get_flops, get_bytes  # noqa: F401\n' \
      "$mod" "$mod" > kernel.py
  timeout 900 python tools/bench.py --kernel "$mod" --json-out "$OUT/refh_$mod.json" > "$OUT/refh_$mod.log" 2>&1
  r=$?; echo "bench $mod rc=$r" >> "$OUT/refh_status.log"; [ $r -ne 0 ] && rc=$r
done
if [ "${3:-}" = ncu ]; then
  printf 'from kernel_opt_agent_b200.qwen35moe_gdn_prefill import KERNEL_TYPE, kernel_fn, get_inputs, get_flops, get_bytes  # noqa: F401\n' > kernel.py
  timeout 600 python tools/ncu_profile.py --kernel-file kernel.py --launch-count 1 \
      --ncu-args "--clock-control none -k regex:gdn_" --output-prefix "$OUT/refh_ncu_gdn" \
      --summary-out "$OUT/refh_ncu_gdn_summary.txt" > "$OUT/refh_ncu_gdn.log" 2>&1
  r=$?; echo "ncu_profile gdn rc=$r" >> "$OUT/refh_status.log"; [ $r -ne 0 ] && rc=$r
fi
rm -rf "$SCRATCH"
exit $rc
