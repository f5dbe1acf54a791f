"""Compare two JSONL benchmark files and flag regressions.

    python benchmarks/compare.py BASE.jsonl NEW.jsonl [--metric max_over_ranks_ms] [--threshold 0.05]

Records are matched on (name, world_size, size, device) (``bench.py`` lines on
metric, n_gpus and impl) and the chosen time metric (lower is better) is compared; when a record carries ``tflops`` or
``gbs`` the throughput ratio is printed next to it.  Exit status 1 when any
matched record is slower than ``1 + threshold`` times its base (a CI gate),
0 otherwise.  The reference ships the same tool
(``benchmarks/compare.py``); the record key and the exit-status contract are
kept so that files written by either harness can be compared.
"""

import argparse
import json
import sys

KEY_FIELDS = ("name", "world_size", "size", "device")


def record_key(rec):
    """(name, world_size, size, device); bench.py lines key on metric, n_gpus and impl."""
    if "name" not in rec and "metric" in rec:
        return (rec["metric"], rec.get("n_gpus"), rec.get("impl", "native"), None)
    return tuple(rec.get(k) for k in KEY_FIELDS)


def load(path):
    out = {}
    with open(path, encoding="utf-8") as f:
        for lineno, line in enumerate(f, 1):
            line = line.strip()
            if not line or not line.startswith("{"):
                continue
            try:
                rec = json.loads(line)
            except ValueError as e:
                raise SystemExit(f"{path}:{lineno}: not JSON: {e}")
            key = record_key(rec)
            out[key] = rec  # a later record of the same key replaces an earlier one
    return out


def time_of(rec, metric):
    for name in (metric, "max_over_ranks_ms", "median_ms", "ms_per_step"):
        if isinstance(rec.get(name), (int, float)):
            return float(rec[name])
    return None


def compare(base, new, metric, threshold):
    rows, regressions = [], 0
    for key in sorted(set(base) | set(new), key=lambda k: tuple(str(x) for x in k)):
        b, n = base.get(key), new.get(key)
        label = "/".join(str(x) for x in key if x is not None)
        if b is None or n is None:
            rows.append((label, "only in " + ("new" if b is None else "base"), "", "", ""))
            continue
        tb, tn = time_of(b, metric), time_of(n, metric)
        if not tb or tn is None:
            rows.append((label, "no time", "", "", ""))
            continue
        ratio = tn / tb
        status = "REGRESSION" if ratio > 1.0 + threshold else ("faster" if ratio < 1.0 - threshold else "same")
        regressions += status == "REGRESSION"
        thr = ""
        for field in ("tflops", "gbs"):
            if b.get(field) and n.get(field):
                thr = f"{field} {n[field] / b[field]:.3f}x"
        rows.append((label, status, f"{tb:.4f}", f"{tn:.4f}", f"{ratio:.3f}" + (f"  {thr}" if thr else "")))
    return rows, regressions


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("base")
    p.add_argument("new")
    p.add_argument("--metric", default="max_over_ranks_ms")
    p.add_argument("--threshold", type=float, default=0.05, help="relative slowdown counted as a regression")
    args = p.parse_args(argv)
    rows, regressions = compare(load(args.base), load(args.new), args.metric, args.threshold)
    width = max([len(r[0]) for r in rows] + [4])
    print(f"{'case':<{width}}  {'status':<10}  {'base_ms':>10}  {'new_ms':>10}  ratio")
    for label, status, tb, tn, ratio in rows:
        print(f"{label:<{width}}  {status:<10}  {tb:>10}  {tn:>10}  {ratio}")
    print(f"{regressions} regression(s) over {args.threshold:.0%}")
    return 1 if regressions else 0


if __name__ == "__main__":
    sys.exit(main())
