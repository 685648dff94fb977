"""Crash -> restart -> resume on GPUs, bit-identical (the elastic configuration, in small).

Two GPU workers train a small bf16 GPT through the restart-all launcher with the
forward+backward CUDA graph and checkpoints every 3 steps.  On the first attempt
rank 1 leaves at step 5 the way the trainer's fault injection does it: between
steps, after synchronising its GPU, so none of its kernels or collectives is in
flight.  Rank 0 finds out through its next collective, whose device-side waits
give up after DTRAIN_TIMEOUT (5 s here) and raise CommError on the host; the
launcher then stops the group and starts a second attempt, which resumes from
the step-3 checkpoint.  The final parameters must equal an uninterrupted run's
bit for bit.  Multicast (NVLS) is not used anywhere in this path.
"""
import os

import pytest
import torch
from harness import max_param_diff, run_job

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
MODEL = ["--dtype", "bfloat16", "--data", "synthetic", "--vocab", "512", "--ctx", "128", "--dim", "128", "--heads",
         "2", "--layers", "2", "--batch", "2", "--steps", "8", "--lr", "3e-3", "--cuda-graph"]


@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["ddp", "zero"])
def test_gpu_crash_restart_resume_is_bit_identical(tmp_path, mode):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    fast = ["--timeout", "5"]
    clean = run_job(tmp_path, mode, 2, MODEL, name="clean", launcher_flags=fast)
    assert clean.code == 0, clean.stderr[-3000:]
    ck = str(tmp_path / "ck")
    crashed = run_job(tmp_path, mode, 2, [*MODEL, "--ckpt-dir", ck, "--ckpt-every", "3", "--resume",
                                          "--fail-at-step", "5", "--fail-rank", "1"],
                      name="crashed", restarts=1, launcher_flags=fast)
    assert crashed.code == 0, crashed.stderr[-4000:]
    assert "injected failure at step 5" in crashed.stderr
    assert "restarting" in crashed.stderr and "resumed from step 3" in crashed.stderr
    assert max_param_diff(crashed.params, clean.params) == 0.0
    losses = [r["loss"] for r in crashed.log if "loss" in r]
    clean_losses = [r["loss"] for r in clean.log if "loss" in r]
    assert losses[-3:] == clean_losses[-3:]  # the resumed steps reproduce the loss trajectory exactly
