"""CPU timing of the reference path (test infrastructure: the CPU-baseline leg of bench.py).

The timed code is the reference's own template inference compiled against
the host Kokkos shim (oracle/_ref/libponni_ref.so, kind "reference") when
that library was built and instantiates the config's network, else the C
port of it (oracle/ponni_oracle.c, kind "port"), which agrees with the
reference bit for bit on the benchmark networks.

Run as a child process so that the OpenMP placement variables reach the
oracle's OpenMP runtime before it starts:

    OMP_NUM_THREADS=<physical cores> OMP_PROC_BIND=spread OMP_PLACES=cores \
        python -m oracle.cpu_bench --config cfg4 [--seconds 10] [--max-cols 1048576]

Protocol: one warm-up call (allocates), then passes over a column slice of
the config's workload (samples are independent, so the per-sample cost does
not depend on the batch), repeated until they total at least `--min-total`
seconds (and at least three passes); the reported rate is the median over
passes.  The slice is sized so that one pass takes about `--seconds` / 4,
within [4096, max_cols] columns.  Prints one JSON object.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="cfg4")
    ap.add_argument("--seconds", type=float, default=10.0, help="approximate budget of the timed passes")
    ap.add_argument("--min-total", type=float, default=1.0)
    ap.add_argument("--max-cols", type=int, default=1 << 20)
    ap.add_argument("--impl", default="auto", choices=["auto", "reference", "port"])
    args = ap.parse_args()

    from ponni_b200 import configs
    from oracle import oracle, ref

    cfg = configs.ALL[args.config](batch=4096)
    threads = int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
    kind = "reference" if args.impl != "port" and ref.available() and ref.network_of(cfg.layers) else "port"
    run = ref.forward if kind == "reference" else oracle.forward
    x = configs.host_inputs(cfg, 4096)
    run(cfg.layers, cfg.dtype, x, nthreads=threads)  # warm-up
    t0 = time.perf_counter()
    run(cfg.layers, cfg.dtype, x, nthreads=threads)
    per_col = max(time.perf_counter() - t0, 1e-6) / 4096
    n = int(min(args.max_cols, max(4096, args.seconds / 4 / per_col)))
    x = configs.host_inputs(cfg, n)
    rates, total = [], 0.0
    while total < args.min_total or len(rates) < 3:
        t0 = time.perf_counter()
        run(cfg.layers, cfg.dtype, x, nthreads=threads)
        dt = time.perf_counter() - t0
        rates.append(n / dt)
        total += dt
        if total > 4 * args.seconds:
            break
    print(json.dumps({"samples_per_s": statistics.median(rates), "columns": n, "passes": len(rates),
                      "seconds": total, "threads": threads, "kind": kind}))


if __name__ == "__main__":
    main()
