"""Training runtime: evaluation, resume and flag handling of the pretraining CLIs (CPU).

* a 2-rank gloo run with the sharded-optimizer engine saves one optimizer
  file per rank, and resuming from the mid-run checkpoint reproduces the
  uninterrupted run's final weights (data position, optimizer shards,
  scheduler and RNG restored);
* ``--eval-every`` evaluates a held-out set, logs ``val/loss`` and keeps
  ``best_model.pt``; fp16 is refused; ``--torch-compile`` on CPU runs eagerly;
* ``--parallel cp`` trains with every sequence split over two gloo ranks;
* ``--parallel pp`` trains MAC as a two-stage pipeline, with checkpoint and resume.
"""

from __future__ import annotations

import json
import os

import pytest
import torch

from tests.test_distributed import run_workers

COMMON = ["--model", "mag", "--dim", "32", "--num-heads", "2", "--num-layers", "2", "--vocab-size", "128",
          "--window-size", "8", "--chunk-size", "16", "--num-persistent-tokens", "2", "--num-memory-layers", "2",
          "--seq-len", "32", "--batch-size", "2", "--mixed-precision", "none", "--num-workers", "0",
          "--log-every", "1", "--synthetic-samples", "64", "--lr", "3e-3"]


def _rank_main(rank, world, argv):
    from titans_pytorch_b200.cli import pretrain_distributed

    pretrain_distributed.main(argv)


def _weights(path):
    return torch.load(path, map_location="cpu", weights_only=False)["model_state_dict"]


def test_distributed_resume_with_optimizer_shards(tmp_path):
    a, b = tmp_path / "a", tmp_path / "b"
    base = COMMON + ["--parallel", "fsdp", "--max-steps", "4", "--eval-every", "0", "--heartbeat-timeout", "30",
                     "--dist-timeout", "60"]
    run_workers(_rank_main, 2, (base + ["--checkpoint-dir", str(a), "--save-every", "2"],), timeout=240)
    mid = a / "step_2.pt"
    assert mid.exists()
    for r in range(2):
        assert (a / f"step_2.pt.optim.rank{r}-of-2").exists()
    ck = torch.load(mid, map_location="cpu", weights_only=False)
    assert ck["optimizer_shards"] == 2 and ck["optimizer_state_dict"] is None and ck["data_position"] == 2
    run_workers(_rank_main, 2, (base + ["--checkpoint-dir", str(b), "--save-every", "0", "--resume", str(mid)],),
                timeout=240)
    wa, wb = _weights(a / "final_model.pt"), _weights(b / "final_model.pt")
    for k in wa:
        torch.testing.assert_close(wb[k], wa[k], rtol=1e-5, atol=1e-6, msg=k)


def test_context_parallel_cli(tmp_path):
    """--parallel cp: two gloo ranks each train on half of every sequence (with evaluation)."""
    ck, mf = tmp_path / "ck", tmp_path / "m.jsonl"
    argv = COMMON + ["--parallel", "cp", "--max-steps", "3", "--eval-every", "2", "--eval-batches", "2",
                     "--save-every", "0", "--checkpoint-dir", str(ck), "--metrics-file", str(mf),
                     "--heartbeat-timeout", "30", "--dist-timeout", "60"]
    run_workers(_rank_main, 2, (argv,), timeout=240)
    lines = [json.loads(x) for x in mf.read_text().splitlines()]
    losses = [x["train/loss"] for x in lines if "train/loss" in x]
    assert losses and all(0 < v < 20 for v in losses)
    assert any("val/loss" in x for x in lines)
    assert (ck / "final_model.pt").exists()


def test_context_parallel_cli_groups(tmp_path):
    """--parallel cp --cp-size 2 on four gloo ranks: two data-parallel replicas of a
    context-parallel pair."""
    ck, mf = tmp_path / "ck", tmp_path / "m.jsonl"
    argv = COMMON + ["--parallel", "cp", "--cp-size", "2", "--max-steps", "2", "--eval-every", "0",
                     "--save-every", "0", "--checkpoint-dir", str(ck), "--metrics-file", str(mf),
                     "--heartbeat-timeout", "30", "--dist-timeout", "60"]
    run_workers(_rank_main, 4, (argv,), timeout=240)
    lines = [json.loads(x) for x in mf.read_text().splitlines()]
    assert [x["step"] for x in lines if "train/loss" in x] == [1, 2]
    assert (ck / "final_model.pt").exists()


def test_pipeline_cli_resume(tmp_path):
    """--parallel pp (MAC over two gloo stages): the checkpoint gathers both stages'
    weights into the model file, keeps one optimizer file per stage, and resuming
    from it reproduces the uninterrupted run."""
    a, b = tmp_path / "a", tmp_path / "b"
    mac = [x if x != "mag" else "mac" for x in COMMON]
    base = mac + ["--parallel", "pp", "--max-steps", "4", "--eval-every", "2", "--eval-batches", "1",
                  "--heartbeat-timeout", "30", "--dist-timeout", "60"]
    run_workers(_rank_main, 2, (base + ["--checkpoint-dir", str(a), "--save-every", "2"],), timeout=240)
    mid = a / "step_2.pt"
    for r in range(2):
        assert (a / f"step_2.pt.optim.rank{r}-of-2").exists()
    wm, wa = _weights(mid), _weights(a / "final_model.pt")
    for blk in (0, 1):  # both stages trained between the two files, and rank 0's files hold both
        k = f"blocks.{blk}.ffn.down_proj.weight"
        assert not torch.allclose(wa[k].float(), wm[k].float()), k
    run_workers(_rank_main, 2, (base + ["--checkpoint-dir", str(b), "--save-every", "0", "--resume", str(mid)],),
                timeout=240)
    wb = _weights(b / "final_model.pt")
    for k in wa:
        torch.testing.assert_close(wb[k], wa[k], rtol=1e-5, atol=1e-6, msg=k)


def test_eval_loop_and_best_model(tmp_path):
    from titans_pytorch_b200.cli import pretrain

    ck, mf = tmp_path / "ck", tmp_path / "m.jsonl"
    pretrain.main(COMMON + ["--max-steps", "4", "--eval-every", "2", "--eval-batches", "2", "--save-every", "0",
                            "--checkpoint-dir", str(ck), "--metrics-file", str(mf)])
    lines = [json.loads(x) for x in mf.read_text().splitlines()]
    vals = [x for x in lines if "val/loss" in x]
    assert [x["step"] for x in vals] == [2, 4]
    assert all(x["val/loss"] > 0 for x in vals)
    assert (ck / "best_model.pt").exists() and (ck / "final_model.pt").exists()
    best = torch.load(ck / "best_model.pt", map_location="cpu", weights_only=False)
    assert best["best_val_loss"] == pytest.approx(min(x["val/loss"] for x in vals))


def test_precision_and_compile_flags(tmp_path, caplog):
    from titans_pytorch_b200.cli import pretrain, pretrain_distributed

    with pytest.raises(SystemExit, match="fp16"):
        pretrain.main(COMMON + ["--mixed-precision", "fp16", "--max-steps", "1"])
    with pytest.raises(SystemExit, match="fp16"):
        pretrain_distributed.main(COMMON + ["--precision", "fp16", "--max-steps", "1"])
    caplog.set_level("INFO")
    pretrain.main(COMMON + ["--max-steps", "1", "--eval-every", "0", "--save-every", "0", "--torch-compile",
                            "--checkpoint-dir", str(tmp_path)])
    assert any("running eagerly" in r.getMessage() for r in caplog.records)
    cmd = pretrain_distributed.relaunch_argv(["--nproc", "4", "--model", "mal", "--nproc=2"], 4, 29500)
    assert cmd[cmd.index("-m") + 1] == "torch.distributed.run" and "--nproc-per-node=4" in cmd
    assert "--nproc" not in cmd and "--nproc=2" not in cmd and cmd[-2:] == ["--model", "mal"]
