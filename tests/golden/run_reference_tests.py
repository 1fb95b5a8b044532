"""Runs the reference's own CPU unit tests under tsrun.py and records the
outcome in reference_unit_tests.json (beside this file).

    python tests/golden/run_reference_tests.py [reference root] [--budget SECONDS] [--workers N]

The reference's golden vectors here (reference_*.npz) come from executing
its TypeScript with tsrun.py; this is the check on the runner itself: the
reference's own test files, whose assertions were written against Bun's
JavaScript engine, run under it with a small `bun:test` (describe / test /
expect). The test files are the reference's, unmodified:

  packages/krystal/src/forward/sampling.test.ts   sampleRow
  packages/krystal/src/host/session.test.ts       packing, think, consider / choose, errors
  packages/krystal/src/host/checkpoint.test.ts    KRY1 write / restore / refusals
  packages/krystal/src/host/learn.test.ts         learn: advantage, critic, rollback, unfreezing
  packages/krystal/src/host/teach.test.ts         teach: showings, forbidden answers, rejection

Each test runs in its own process with a time budget: the runner executes
the model at Python speed, and some learn tests train for hundreds of
rounds, which is hours here; a test stopped by its budget is recorded as not
run, not as passed. (The WebGPU tests under packages/webgpu/test need a
WebGPU device and are not run.) tests/test_reference_golden.py reads the
record.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import sys
import time
from concurrent.futures import ProcessPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import tsrun  # noqa: E402

FILES = ("forward/sampling.test.ts", "host/session.test.ts", "host/checkpoint.test.ts", "host/learn.test.ts",
         "host/teach.test.ts")


def _run(path: str, select, budget_s):
    results = []
    runner = tsrun.Runner(packages={"bun:test": tsrun.bun_test_module(results, select, budget_s)})
    runner.load(Path(path))
    return results


def _one(args):
    path, k, budget_s = args
    t0 = time.time()
    results = _run(path, {k}, budget_s)
    name, err = results[k]
    return k, name, err, time.time() - t0


def main():
    args = sys.argv[1:]
    budget, workers = 1200, 8
    for flag in ("--budget", "--workers"):
        if flag in args:
            i = args.index(flag)
            if flag == "--budget":
                budget = int(args[i + 1])
            else:
                workers = int(args[i + 1])
            del args[i:i + 2]
    root = Path(args[0]) if args else Path("/root/reference")
    jobs, names = [], {}
    for f in FILES:
        path = str(root / "packages/krystal/src" / f)
        listed = _run(path, set(), None)  # declares every test, runs none
        names[f] = [n for n, _ in listed]
        jobs += [(f, path, k) for k in range(len(listed))]
    record = {f: [None] * len(n) for f, n in names.items()}
    with ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as pool:
        futures = {pool.submit(_one, (path, k, budget)): (f, k) for f, path, k in jobs}
        for fut in futures:
            f, k = futures[fut]
            _, name, err, secs = fut.result()
            status = "passed" if err is None else ("not run" if err.startswith("out of time") else "failed")
            record[f][k] = {"test": name, "status": status, "error": err, "seconds": round(secs, 1)}
            print(f"{f} #{k} {status} ({secs:.0f} s): {name}" + (f" -- {err}" if err else ""), flush=True)
    (HERE / "reference_unit_tests.json").write_text(json.dumps(record, indent=1) + "\n")


if __name__ == "__main__":
    main()
