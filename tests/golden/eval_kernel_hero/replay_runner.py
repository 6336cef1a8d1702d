#!/usr/bin/env python3
"""Replays what bin/custom_runner printed on a B200 for the hero dataset (test fixture).

tests/test_runner_gpu.py::test_hero_dataset_through_eval_kernel_invocations runs custom_runner
on configs/fixed_bf16_gemm_v1.json's three cases with the argv scripts/eval_kernel.py builds
(run_runner :316-340) and, with MO_EVK_RECORD set, keeps each JSON result and its argv here.
This script takes the runner's command line, checks that its flags are the recorded ones (paths
aside), and writes the recorded JSON to --json-out, so that the reference's own eval_kernel.py can
be run on a machine without a GPU against the outputs the real runner produced.
"""

import argparse
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> int:
    ap = argparse.ArgumentParser()
    for flag in ("--dataset-dir", "--case-id", "--mode", "--warmup", "--iters", "--flush-cache-mb", "--json-out"):
        ap.add_argument(flag, required=True)
    args, extra = ap.parse_known_args()
    stem = f"{args.mode}_{args.case_id}"
    recorded = HERE / f"{stem}.json"
    if not recorded.exists():
        sys.stderr.write(f"no recorded run for {stem}\n")
        return 1
    want = json.loads((HERE / f"{stem}.argv.json").read_text())
    got = ["--dataset-dir", "<dataset-dir>", "--case-id", args.case_id, "--mode", args.mode,
           "--warmup", args.warmup, "--iters", args.iters, "--flush-cache-mb", args.flush_cache_mb,
           "--json-out", "<json-out>", *extra]
    if got != want:
        sys.stderr.write(f"argv differs from the recorded run: {got} != {want}\n")
        return 1
    Path(args.json_out).write_text(recorded.read_text())
    return 0


if __name__ == "__main__":
    sys.exit(main())
