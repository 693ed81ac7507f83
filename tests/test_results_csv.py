"""The results/*.csv wire format of the sweep tool against the reference's column orders
(results/steps_per_sec.csv, pendulum.csv, aba.csv, legged.csv and es*.csv headers, written by
bench.py:96-101, bench_pendulum.py:129-133, bench_legged.py:78-82 and bench_ppo.py:37-41).
The CPU tests write fabricated rows; the GPU tests run a tiny sweep end to end."""

import csv

import pytest

import bench_sweep

HEADERS = {
    "steps_per_sec.csv": "config,n,steps_per_sec,iters,warmup,repeats",
    "pendulum.csv": "k,config,n,steps_per_sec,iters,warmup,repeats",
    "aba.csv": "k,config,n,steps_per_sec,iters,warmup,repeats",
    "legged.csv": "c,config,n,steps_per_sec,sweeps,iters,warmup,repeats",
    "es.csv": "backend,lr,series,n,seed,solved,generations,env_steps,train_seconds,score,steps_per_sec",
}


def _lines(path):
    return path.read_text().splitlines()


def test_step_writers_match_reference_columns(tmp_path):
    plain = [{"config": "cuda kernel, sync every 32", "n": 1, "steps_per_sec": 123}]
    bench_sweep.write_steps_csv(plain, tmp_path / "a.csv", 256, 16, 3)
    assert _lines(tmp_path / "a.csv") == [HEADERS["steps_per_sec.csv"], '"cuda kernel, sync every 32",1,123,256,16,3']
    keyed = [{"k": 8, "config": "x", "n": 4, "steps_per_sec": 9}]
    bench_sweep.write_steps_csv(keyed, tmp_path / "b.csv", 64, 8, 3)
    assert _lines(tmp_path / "b.csv") == [HEADERS["pendulum.csv"], "8,x,4,9,64,8,3"]
    legs = [{"c": 4, "config": "x", "n": 2, "steps_per_sec": 7}]
    bench_sweep.write_steps_csv(legs, tmp_path / "c.csv", 64, 8, 3, sweeps=8)
    assert _lines(tmp_path / "c.csv") == [HEADERS["legged.csv"], "4,x,2,7,8,64,8,3"]


def test_es_writer_matches_reference_columns(tmp_path):
    row = {"backend": "cuda", "lr": 0.1, "series": "cuda", "n": 64, "seed": 0, "solved": True, "generations": 3,
           "env_steps": 100, "train_seconds": 0.5, "score": 500.0, "steps_per_sec": 200.0}
    bench_sweep.write_dict_csv([row], tmp_path / "es.csv")
    got = list(csv.reader(open(tmp_path / "es.csv")))
    assert ",".join(got[0]) == HEADERS["es.csv"] and got[1][0] == "cuda" and got[1][5] == "True"


def test_es_rows_take_result_fields_in_order():
    """The ES row is backend, lr, series, n, seed, then the training result's fields, then
    steps_per_sec: the result must carry exactly the reference's fields, in its order."""
    import dataclasses

    import es

    assert [f.name for f in dataclasses.fields(es.Result)] == ["solved", "generations", "env_steps", "train_seconds", "score"]
    assert bench_sweep.ES_COLUMNS == HEADERS["es.csv"].split(",")


def test_file_names_and_defaults_follow_the_reference():
    assert {b: f for b, (f, _) in bench_sweep.STEP_FILES.items()}["cartpole"] == "steps_per_sec.csv"
    assert set(HEADERS) - {"es.csv"} <= {f for f, _ in bench_sweep.STEP_FILES.values()}
    a = bench_sweep._parse(["steps", "--body", "legged"])
    assert a.cs == [1, 2, 4] and a.sweeps == 8 and a.repeats == 3 and a.eval_every == 32
    e = bench_sweep._parse(["es"])
    assert e.ns == [64, 256, 1024, 4096, 16384, 65536] and e.seeds == [0, 1, 2, 3, 4] and e.sigma == 0.1


@pytest.mark.gpu
@pytest.mark.parametrize("body,extra", [("cartpole", []), ("acrobot", []), ("hopper", []),
                                        ("pendulum", ["--ks", "4"]), ("aba", ["--ks", "8"]),
                                        ("legged", ["--cs", "2"])])
def test_tiny_sweep_writes_reference_csv(cuda, tmp_path, body, extra):
    path = bench_sweep.main(["--results", str(tmp_path), "steps", "--body", body, "--max-exp", "3", "--iters", "4",
                             "--warmup", "1", "--repeats", "1", "--eval-every", "2", *extra])
    rows = list(csv.DictReader(open(path)))
    assert _lines(path)[0] == HEADERS.get(path.name, HEADERS["steps_per_sec.csv"])
    assert len(rows) == 4 * len({r["config"] for r in rows}) and all(int(r["steps_per_sec"]) > 0 for r in rows)


@pytest.mark.gpu
def test_tiny_es_sweep_writes_reference_csv(cuda, tmp_path):
    path = bench_sweep.main(["--results", str(tmp_path), "es", "--task", "cartpole", "--ns", "64", "--seeds", "0",
                             "--max-generations", "2", "--time-budget", "30"])
    assert path.name == "es.csv" and _lines(path)[0] == HEADERS["es.csv"]
    rows = list(csv.DictReader(open(path)))
    assert len(rows) == 1 and int(rows[0]["generations"]) >= 1 and float(rows[0]["steps_per_sec"]) > 0
