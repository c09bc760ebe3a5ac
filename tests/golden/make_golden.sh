#!/usr/bin/env bash
# Regenerates tests/golden/pkt_train_linear_cpu.txt from Marco-Christiani/pkt's
# own train_linear binary (built by `make -C oracle ref` from the reference
# sources). Only the host part runs here: pkt prints its CPU-loop results
# (examples/train_linear.cu:380-415) before its first device allocation, which
# fails on a machine without a GPU. Run in the build container, not on the GPU box.
set -u
HERE="$(cd "$(dirname "$0")" && pwd)"
BIN="$HERE/../../oracle/_ref/train_linear"
OUT="$HERE/pkt_train_linear_cpu.txt"
: > "$OUT"
run() {
  echo "### args: $*" >> "$OUT"
  "$BIN" "$@" 2>/dev/null | grep -E '^(Initial host loss|CPU final loss|CPU first step loss|x\[0:5\]|target\[0:5\]|Host expected y\[0\])' >> "$OUT"
}
run --m 64 --n 128 --batch 256 --steps 100 --lr 0.01
run --m 128 --n 64 --batch 64 --steps 20 --lr 0.01
run --m 32 --n 48 --batch 16 --steps 7 --lr 0.05
run --m 256 --n 256 --batch 32 --steps 5 --lr 0.001
