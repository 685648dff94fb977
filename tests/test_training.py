"""End-to-end distributed training through the launcher (real processes, fp64 CPU ranks).

Same checks as the reference's integration tests, plus equality with the
reference's own training run and checkpoint-format compatibility with it.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

PY = sys.executable
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
TINY = ["--dim", "16", "--heads", "2", "--layers", "2", "--ctx", "16", "--batch", "2", "--dtype", "float64",
        "--lr", "3e-3", "--warmup", "2"]


@pytest.fixture(scope="module")
def corpus(tmp_path_factory):
    rng = np.random.default_rng(0)
    words = ["the", "king", "and", "queen", "of", "rome", "said", "to", "thee", "now"]
    p = tmp_path_factory.mktemp("data") / "corpus.txt"
    p.write_text(" ".join(rng.choice(words, 4000)) + "\n")
    return str(p)


def train(tmp, name, corpus, mode, nproc=1, extra=(), restarts=0, check=True, pkg="dtrain_b200"):
    out = tmp / f"{name}.npz"
    log = tmp / f"{name}.jsonl"
    args = ["-m", f"{pkg}.train", "--mode", mode, "--data", corpus, "--save-params", str(out), "--log", str(log),
            *TINY, *extra]
    if mode == "single":
        cmd = [PY, *args]
    else:
        cmd = [PY, "-m", f"{pkg}.launch", "--nproc", str(nproc), "--max-restarts", str(restarts), "--timeout", "30",
               "--", PY, *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1",
               PYTHONPATH=(REF if pkg == "dtrain" else ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    if check:
        assert r.returncode == 0, r.stderr[-3000:]
    params = dict(np.load(out)) if out.exists() else None
    logs = [json.loads(line) for line in open(log)] if log.exists() else []
    return params, logs, r


def assert_close(a, b, tol):
    assert a.keys() == b.keys()
    worst = max(float(np.max(np.abs(a[k] - b[k]))) for k in a)
    assert worst <= tol, f"max abs param difference {worst:g} > {tol:g}"


STEPS = ["--steps", "6"]
needs_ref = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "dtrain")), reason="reference not installed")


def test_ddp_matches_single_process(tmp_path, corpus):
    ref, ref_log, _ = train(tmp_path, "single", corpus, "single", extra=[*STEPS, "--emulate-world", "4"])
    ddp, ddp_log, _ = train(tmp_path, "ddp", corpus, "ddp", 4, extra=STEPS)
    assert_close(ddp, ref, 1e-10)
    for a, b in zip(ref_log, ddp_log):
        assert abs(a["loss"] - b["loss"]) < 1e-10


def test_zero_matches_ddp_and_shards_state(tmp_path, corpus):
    ddp, _, _ = train(tmp_path, "ddp", corpus, "ddp", 4, extra=STEPS)
    zero, zlog, _ = train(tmp_path, "zero", corpus, "zero", 4, extra=STEPS)
    assert_close(zero, ddp, 1e-10)
    nparams = sum(v.size for v in ddp.values())
    state = [x for x in zlog if "optimizer_state_bytes_per_rank" in x][0]["optimizer_state_bytes_per_rank"]
    assert state == 2 * 8 * -(-nparams // 4)  # rank 0: m and v (float64) for ceil(n/4) elements


def test_overlap_bucket_size_and_algorithm_do_not_change_results(tmp_path, corpus):
    a, _, _ = train(tmp_path, "a", corpus, "ddp", 3, extra=[*STEPS, "--bucket-mb", "0.001"])
    b, _, _ = train(tmp_path, "b", corpus, "ddp", 3, extra=[*STEPS, "--no-overlap", "--bucket-mb", "100"])
    c, _, _ = train(tmp_path, "c", corpus, "ddp", 3, extra=[*STEPS, "--algo", "direct"])
    assert_close(a, b, 1e-12)
    assert_close(a, c, 1e-12)


def test_gradient_accumulation_matches_larger_batch(tmp_path, corpus):
    ref, _, _ = train(tmp_path, "ref", corpus, "single", extra=[*STEPS, "--emulate-world", "2", "--accum", "2"])
    ddp, _, _ = train(tmp_path, "acc", corpus, "ddp", 2, extra=[*STEPS, "--accum", "2"])
    assert_close(ddp, ref, 1e-10)


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_checkpoint_resume_is_exact(tmp_path, corpus, mode):
    full, _, _ = train(tmp_path, f"{mode}-full", corpus, mode, 2, extra=["--steps", "8"])
    ck = tmp_path / f"ck-{mode}"
    train(tmp_path, f"{mode}-part", corpus, mode, 2,
          extra=["--steps", "8", "--stop-after", "4", "--ckpt-dir", str(ck), "--ckpt-every", "2"])
    resumed, _, r = train(tmp_path, f"{mode}-res", corpus, mode, 2,
                          extra=["--steps", "8", "--ckpt-dir", str(ck), "--ckpt-every", "2", "--resume"])
    assert "resumed from step 4" in r.stderr
    assert_close(resumed, full, 0.0)


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_worker_crash_restart_resume_matches_failure_free_run(tmp_path, corpus, mode):
    clean, _, _ = train(tmp_path, f"{mode}-clean", corpus, mode, 3, extra=["--steps", "9"])
    ck = tmp_path / f"ck-fail-{mode}"
    crashed, _, r = train(tmp_path, f"{mode}-crash", corpus, mode, 3, restarts=2,
                          extra=["--steps", "9", "--ckpt-dir", str(ck), "--ckpt-every", "3", "--resume",
                                 "--fail-at-step", "5", "--fail-rank", "1"])
    assert "injected failure at step 5" in r.stderr
    assert "restarting" in r.stderr and "resumed from step 3" in r.stderr
    assert_close(crashed, clean, 0.0)


def test_no_restarts_left_propagates_failure(tmp_path, corpus):
    _, _, r = train(tmp_path, "fail", corpus, "ddp", 2, restarts=0, check=False,
                    extra=["--steps", "4", "--fail-at-step", "1", "--fail-rank", "0"])
    assert r.returncode == 17


def test_corrupt_checkpoint_is_rejected(tmp_path, corpus):
    ck = tmp_path / "ck-bad"
    train(tmp_path, "w", corpus, "ddp", 2, extra=["--steps", "2", "--ckpt-dir", str(ck), "--ckpt-every", "2"])
    shard = ck / "step_000002" / "rank1.npz"
    b = bytearray(shard.read_bytes())
    b[len(b) // 2] ^= 0xFF
    shard.write_bytes(bytes(b))
    _, _, r = train(tmp_path, "r", corpus, "ddp", 2, check=False,
                    extra=["--steps", "4", "--ckpt-dir", str(ck), "--resume"])
    assert r.returncode != 0 and "checksum mismatch" in r.stderr


@needs_ref
@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_matches_the_reference_training_run(tmp_path, corpus, mode):
    ours, our_log, _ = train(tmp_path, f"ours-{mode}", corpus, mode, 2, extra=STEPS)
    ref, ref_log, _ = train(tmp_path, f"ref-{mode}", corpus, mode, 2, extra=STEPS, pkg="dtrain")
    assert_close(ours, ref, 1e-10)
    for a, b in zip(our_log, ref_log):
        if "loss" in a:
            assert abs(a["loss"] - b["loss"]) < 1e-10


@needs_ref
@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_checkpoints_interchange_with_the_reference(tmp_path, corpus, mode):
    """Our checkpoint resumes in the reference and the reference's resumes here, bit-exactly."""
    full, _, _ = train(tmp_path, f"full-{mode}", corpus, mode, 2, extra=["--steps", "6"])
    ck = tmp_path / f"ck-x-{mode}"
    train(tmp_path, f"part-{mode}", corpus, mode, 2,
          extra=["--steps", "6", "--stop-after", "3", "--ckpt-dir", str(ck), "--ckpt-every", "3"])
    res_ref, _, r = train(tmp_path, f"res-ref-{mode}", corpus, mode, 2, pkg="dtrain",
                          extra=["--steps", "6", "--ckpt-dir", str(ck), "--resume"])
    assert "resumed from step 3" in r.stderr
    assert_close(res_ref, full, 1e-12)
    ck2 = tmp_path / f"ck-y-{mode}"
    train(tmp_path, f"part2-{mode}", corpus, mode, 2, pkg="dtrain",
          extra=["--steps", "6", "--stop-after", "3", "--ckpt-dir", str(ck2), "--ckpt-every", "3"])
    res_ours, _, r = train(tmp_path, f"res-ours-{mode}", corpus, mode, 2,
                           extra=["--steps", "6", "--ckpt-dir", str(ck2), "--resume"])
    assert "resumed from step 3" in r.stderr
    assert_close(res_ours, full, 1e-12)


def test_precision_flag_is_a_short_form_of_dtype():
    from dtrain_b200 import train as T
    assert T.parse(["--precision", "bf16"]).dtype == "bfloat16"
    assert T.parse(["--precision", "fp64"]).dtype == "float64"
    assert T.parse(["--dtype", "float32"]).dtype == "float32"


@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_async_checkpoints_match_synchronous_ones(tmp_path, corpus, mode):
    """--async-ckpt writes the same shard files (same bytes) and commits them in the same
    layout; resuming from one reproduces the uninterrupted run exactly."""
    full, _, _ = train(tmp_path, f"{mode}-full", corpus, mode, 2, extra=["--steps", "8"])
    sync_ck, async_ck = tmp_path / f"sync-{mode}", tmp_path / f"async-{mode}"
    train(tmp_path, f"{mode}-sync", corpus, mode, 2,
          extra=["--steps", "8", "--stop-after", "4", "--ckpt-dir", str(sync_ck), "--ckpt-every", "2"])
    train(tmp_path, f"{mode}-async", corpus, mode, 2,
          extra=["--steps", "8", "--stop-after", "4", "--ckpt-dir", str(async_ck), "--ckpt-every", "2",
                 "--async-ckpt"])
    for step in ("step_000002", "step_000004"):
        for f in ("rank0.npz", "rank1.npz", "manifest.json"):
            assert (sync_ck / step / f).read_bytes() == (async_ck / step / f).read_bytes(), (step, f)
    assert (async_ck / "LATEST").read_text() == "step_000004"
    resumed, _, r = train(tmp_path, f"{mode}-res", corpus, mode, 2,
                          extra=["--steps", "8", "--ckpt-dir", str(async_ck), "--ckpt-every", "2", "--resume",
                                 "--async-ckpt"])
    assert "resumed from step 4" in r.stderr
    assert_close(resumed, full, 0.0)
