"""Experiments benchmark grid: CSV layout, ranking rule, and one real CPU grid run of the trainer."""
import csv

from hrm_flashrenderer_b200.experiments import bench_cli


def _write(path, rows):
    with open(path, "w", newline="") as f:
        f.write("runner,scenario,lr,rep,tok_s,elapsed_sec\n")
        for r in rows:
            f.write(",".join(str(x) for x in r) + "\n")


def test_ranking_rule(tmp_path):
    p = tmp_path / "raw.csv"
    _write(p, [("a", "s1", "0.001", 1, 100, 10), ("a", "s2", "0.001", 1, 100, 10),
               ("b", "s1", "0.001", 1, 200, 20), ("b", "s2", "0.001", 1, 50, 20),
               ("c", "s1", "0.001", 1, 150, 10), ("c", "s2", "0.001", 1, 160, 10),
               ("d", "s1", "0.001", 1, "NA", "NA")])
    scored, winner = bench_cli.summarize(p)
    keys = {k: (score, mt, ms, w) for score, k, mt, ms, tot, w in scored}
    assert set(keys) == {"a@0.001", "b@0.001", "c@0.001"}          # failed runs are skipped
    # mean tok/s a 100, b 125, c 155 (min-max: 0, 25/55, 1); mean time a 10, b 20, c 10 (0, 1, 0);
    # wins: s1 -> b, s2 -> c
    assert abs(keys["a@0.001"][0] - 0.0) < 1e-9
    assert abs(keys["b@0.001"][0] - (25 / 55 - 1 + 0.08)) < 1e-9
    assert abs(keys["c@0.001"][0] - 1.08) < 1e-9
    assert winner == "c@0.001"


def test_normalize_lr_and_presets():
    assert bench_cli.normalize_lr(0.0003) == "0.0003" and bench_cli.normalize_lr(1e-3) == "0.001"
    assert [s[0] for s in bench_cli.PRESETS["decision"]] == ["shakespeare", "code", "german", "shakespeare_long"]


def test_cpu_grid_run(tmp_path, capsys):
    extra = "--device cpu --k1 64 --k2 32 --dmodel 32 --heads 2 --layers 1 --ffn 48 --tmax 64"
    rc = bench_cli.main(["--preset", "matrix", "--repeats", "1", "--steps", "4", "--log-every", "2",
                         "--lr-list", "0.001", "--runners", "revlm_eager", "--out", str(tmp_path), "--extra", extra])
    assert rc == 0
    rows = list(csv.DictReader(open(tmp_path / "raw.csv")))
    assert [r["scenario"] for r in rows] == ["shakespeare", "code", "german"]
    assert all(float(r["tok_s"]) > 0 and float(r["elapsed_sec"]) > 0 for r in rows)
    assert "WINNER: revlm_eager@0.001" in capsys.readouterr().out
