"""Training jobs end to end: CLI, launcher, real processes, fp64 CPU ranks.

Pinned behaviours (the reference's integration tests, tests/test_training.py there):
data-parallel and ZeRO-1 jobs reproduce a single process that emulates the same
global batch; bucket size, overlap and summation order leave the result unchanged;
gradient accumulation equals the larger batch; stop/resume and crash/restart/resume
are bit-identical to an uninterrupted run; an injected crash with no restart left
surfaces exit code 17; a corrupted shard is refused.  Added here: equality with the
reference's own training run, checkpoint interchange with it in both directions,
asynchronous checkpoints, and the launcher's per-attempt exit records.
"""
import json

import pytest
from harness import HAVE_REF, max_param_diff, run_job

MODEL = ["--dim", "24", "--heads", "2", "--layers", "2", "--ctx", "12", "--batch", "3", "--dtype", "float64",
         "--lr", "2e-3", "--warmup", "2"]
STEPS = 5


@pytest.fixture(scope="module")
def jobs(tmp_path_factory, corpus):
    """Runs each distinct (mode, world, flags) job once per module."""
    workdir = tmp_path_factory.mktemp("jobs")
    cache = {}

    def get(mode, world, *flags, steps=STEPS):
        key = (mode, world, flags, steps)
        if key not in cache:
            name = f"{mode}{world}-{len(cache)}"
            job = run_job(workdir, mode, world, ["--data", corpus, "--steps", str(steps), *MODEL, *flags], name=name)
            assert job.code == 0, job.stderr[-3000:]
            cache[key] = job
        return cache[key]

    return get


# (description, job A, job B, max |param difference|)
EQUIVALENT = [
    ("ddp on 4 ranks == one process emulating 4 ranks", ("ddp", 4), ("single", 1, "--emulate-world", "4"), 1e-10),
    ("zero on 4 ranks == ddp on 4 ranks", ("zero", 4), ("ddp", 4), 1e-10),
    ("1 KiB buckets overlapped == one 100 MiB bucket after backward",
     ("ddp", 3, "--bucket-mb", "0.001"), ("ddp", 3, "--no-overlap", "--bucket-mb", "100"), 1e-12),
    ("ring order == direct order", ("ddp", 3), ("ddp", 3, "--algo", "direct"), 1e-12),
    ("2 micro-steps on 2 ranks == one process emulating 2 ranks with 2 micro-steps",
     ("ddp", 2, "--accum", "2"), ("single", 1, "--emulate-world", "2", "--accum", "2"), 1e-10),
]


@pytest.mark.parametrize("case", EQUIVALENT, ids=[c[0] for c in EQUIVALENT])
def test_equivalent_jobs_train_the_same_model(jobs, case):
    _, a, b, tol = case
    ja, jb = jobs(*a), jobs(*b)
    assert max_param_diff(ja.params, jb.params) <= tol
    la = [r["loss"] for r in ja.log if "loss" in r]
    lb = [r["loss"] for r in jb.log if "loss" in r]
    assert len(la) == len(lb) == STEPS
    assert max(abs(x - y) for x, y in zip(la, lb)) <= 1e-10


def test_zero_keeps_one_shard_of_optimizer_state_per_rank(jobs):
    ddp, zero = jobs("ddp", 4), jobs("zero", 4)
    n = sum(v.size for v in ddp.params.values())
    rec = [r for r in zero.log if "optimizer_state_bytes_per_rank" in r]
    assert rec and rec[0]["optimizer_state_bytes_per_rank"] == 2 * 8 * -(-n // 4)  # rank 0: fp64 m and v


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_preempted_job_resumes_bit_identically(tmp_path, corpus, mode):
    common = ["--data", corpus, "--steps", "7", *MODEL]
    whole = run_job(tmp_path, mode, 2, common, name="whole")
    ck = str(tmp_path / "ck")
    first = run_job(tmp_path, mode, 2, [*common, "--stop-after", "4", "--ckpt-dir", ck, "--ckpt-every", "2"],
                    name="first")
    second = run_job(tmp_path, mode, 2, [*common, "--ckpt-dir", ck, "--ckpt-every", "2", "--resume"], name="second")
    assert whole.code == first.code == second.code == 0, second.stderr[-2000:]
    assert "resumed from step 4" in second.stderr
    assert max_param_diff(second.params, whole.params) == 0.0


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_crash_restart_resume_is_bit_identical(tmp_path, corpus, mode):
    common = ["--data", corpus, "--steps", "8", *MODEL]
    clean = run_job(tmp_path, mode, 3, common, name="clean")
    ck = str(tmp_path / "ck")
    exits = str(tmp_path / "exits.jsonl")
    crashed = run_job(tmp_path, mode, 3, [*common, "--ckpt-dir", ck, "--ckpt-every", "2", "--resume",
                                          "--fail-at-step", "5", "--fail-rank", "2"],
                      name="crashed", restarts=1, launcher_flags=["--exit-log", exits])
    assert clean.code == crashed.code == 0, crashed.stderr[-3000:]
    assert "injected failure at step 5" in crashed.stderr
    assert "exited with" in crashed.stderr and "restarting" in crashed.stderr
    assert "resumed from step 4" in crashed.stderr
    assert max_param_diff(crashed.params, clean.params) == 0.0
    recs = [json.loads(line) for line in open(exits)]
    first = {r["rank"]: r for r in recs if r["attempt"] == 0}
    assert set(first) == {0, 1, 2}
    assert (first[2]["code"], first[2]["cause"]) == (17, "failed")  # the injected crash
    # the survivors either noticed the dead peer themselves or were stopped by the launcher
    assert all(first[r]["cause"] in ("failed", "stopped") and first[r]["code"] != 0 for r in (0, 1))
    assert sorted((r["rank"], r["code"], r["cause"]) for r in recs if r["attempt"] == 1) == [
        (0, 0, "ok"), (1, 0, "ok"), (2, 0, "ok")]


def test_failure_without_restarts_returns_the_workers_code(tmp_path, corpus):
    job = run_job(tmp_path, "ddp", 2, ["--data", corpus, "--steps", "4", *MODEL, "--fail-at-step", "2",
                                       "--fail-rank", "1"], name="fail")
    assert job.code == 17
    assert "injected failure at step 2" in job.stderr


def test_corrupted_shard_is_refused(tmp_path, corpus):
    ck = tmp_path / "ck"
    common = ["--data", corpus, *MODEL, "--ckpt-dir", str(ck)]
    assert run_job(tmp_path, "ddp", 2, [*common, "--steps", "2", "--ckpt-every", "2"], name="w").code == 0
    shard = ck / "step_000002" / "rank0.npz"
    data = bytearray(shard.read_bytes())
    data[-len(data) // 3] ^= 0x5A
    shard.write_bytes(bytes(data))
    job = run_job(tmp_path, "ddp", 2, [*common, "--steps", "4", "--resume"], name="r")
    assert job.code != 0 and "checksum mismatch" in job.stderr


needs_ref = pytest.mark.skipif(not HAVE_REF, reason="reference not installed in baseline/_ref")


@needs_ref
@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_matches_the_reference_training_run(tmp_path, corpus, mode):
    flags = ["--data", corpus, "--steps", str(STEPS), *MODEL]
    ours = run_job(tmp_path, mode, 2, flags, name="ours")
    ref = run_job(tmp_path, mode, 2, flags, name="ref", package="dtrain")
    assert ours.code == ref.code == 0
    assert max_param_diff(ours.params, ref.params) <= 1e-10
    for a, b in zip(ours.log, ref.log):
        if "loss" in a:
            assert abs(a["loss"] - b["loss"]) < 1e-10


@needs_ref
@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_checkpoints_interchange_with_the_reference(tmp_path, corpus, mode):
    """A checkpoint written here resumes in the reference, and one written by the
    reference resumes here, both reproducing the uninterrupted run."""
    common = ["--data", corpus, "--steps", "6", *MODEL]
    full = run_job(tmp_path, mode, 2, common, name="full")
    for writer, reader in (("dtrain_b200", "dtrain"), ("dtrain", "dtrain_b200")):
        ck = str(tmp_path / f"ck-{writer}")
        run_job(tmp_path, mode, 2, [*common, "--stop-after", "3", "--ckpt-dir", ck, "--ckpt-every", "3"],
                name=f"w-{writer}", package=writer)
        res = run_job(tmp_path, mode, 2, [*common, "--ckpt-dir", ck, "--resume"], name=f"r-{reader}", package=reader)
        assert res.code == 0 and "resumed from step 3" in res.stderr, res.stderr[-2000:]
        assert max_param_diff(res.params, full.params) <= 1e-12


def test_precision_flag_is_a_short_form_of_dtype():
    from dtrain_b200 import train as T
    assert T.parse(["--precision", "bf16"]).dtype == "bfloat16"
    assert T.parse(["--precision", "fp64"]).dtype == "float64"
    assert T.parse(["--dtype", "float32"]).dtype == "float32"


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_async_checkpoints_match_synchronous_ones(tmp_path, corpus, mode):
    """--async-ckpt writes the same shard files (same bytes) and commits them in the same
    layout; resuming from one reproduces the uninterrupted run exactly."""
    common = ["--data", corpus, "--steps", "8", *MODEL]
    full = run_job(tmp_path, mode, 2, common, name="full")
    sync_ck, async_ck = tmp_path / "sync", tmp_path / "async"
    run_job(tmp_path, mode, 2, [*common, "--stop-after", "4", "--ckpt-dir", str(sync_ck), "--ckpt-every", "2"],
            name="sync")
    run_job(tmp_path, mode, 2, [*common, "--stop-after", "4", "--ckpt-dir", str(async_ck), "--ckpt-every", "2",
                                "--async-ckpt"], name="async")
    for step in ("step_000002", "step_000004"):
        for f in ("rank0.npz", "rank1.npz", "manifest.json"):
            assert (sync_ck / step / f).read_bytes() == (async_ck / step / f).read_bytes(), (step, f)
    assert (async_ck / "LATEST").read_text() == "step_000004"
    res = run_job(tmp_path, mode, 2, [*common, "--ckpt-dir", str(async_ck), "--ckpt-every", "2", "--resume",
                                      "--async-ckpt"], name="res")
    assert "resumed from step 4" in res.stderr
    assert max_param_diff(res.params, full.params) == 0.0
