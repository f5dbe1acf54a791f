import json
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "benchmarks"))
import compare  # noqa: E402


def _write(path, records):
    with open(path, "w") as f:
        for r in records:
            f.write(json.dumps(r) + "\n")


def test_compare_flags_regressions(tmp_path, capsys):
    base, new = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    common = {"world_size": 2, "size": "small", "device": "cpu"}
    _write(base, [dict(common, name="x", max_over_ranks_ms=1.0), dict(common, name="y", max_over_ranks_ms=2.0),
                  dict(common, name="gone", max_over_ranks_ms=1.0)])
    _write(new, [dict(common, name="x", max_over_ranks_ms=1.2), dict(common, name="y", max_over_ranks_ms=1.0),
                 dict(common, name="added", max_over_ranks_ms=1.0)])
    assert compare.main([str(base), str(new)]) == 1
    out = capsys.readouterr().out
    assert "REGRESSION" in out and "faster" in out and "only in base" in out and "only in new" in out
    assert compare.main([str(base), str(new), "--threshold", "0.25"]) == 0


def test_compare_reads_bench_lines(tmp_path):
    base, new = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    line = {"metric": "TP-contraction TFLOP/s", "n_gpus": 1, "impl": "native", "value": 1300.0}
    _write(base, [dict(line, ms_per_step=70.0)])
    _write(new, [dict(line, ms_per_step=80.0)])
    assert compare.main([str(base), str(new)]) == 1
    _write(new, [dict(line, ms_per_step=70.5)])
    assert compare.main([str(base), str(new)]) == 0
