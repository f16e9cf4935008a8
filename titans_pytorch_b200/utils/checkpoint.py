"""Checkpoints in the reference's formats.

The reference's loaders (`scripts/inference.py:130-165`,
`scripts/eval_perplexity.py:87-94`, `scripts/benchmark_babilong.py:104-111`)
read ``TitansConfig(**ckpt["config"])``, ``ckpt["model_type"]`` and
``ckpt["model_state_dict"]``.  :func:`save_checkpoint` writes exactly that (the
config restricted to the reference's fields, the tied ``head.weight`` present
as in ``state_dict()``), plus the training state the reference's trainer
stores (`scripts/pretrain.py:657-672`: optimizer, scheduler, scaler, step,
epoch, best val loss) and the resume extras it lacks (RNG states, data
position).  :func:`load_checkpoint` also reads the reference's own trainer
checkpoints, whose ``config`` is the trainer's flag dict and which have no
``model_type`` (inferred from the state-dict keys), and strips the
``_orig_mod.`` prefix torch.compile leaves on keys.
"""

from __future__ import annotations

import os
import random
from typing import Any

import numpy as np
import torch

from ..config import TitansConfig
from ..models.titans import MODEL_CLASSES


def infer_model_type(state_dict: dict[str, torch.Tensor]) -> str:
    keys = state_dict.keys()
    if any(".norm_mem." in k for k in keys):
        return "mac"
    if any(".norm3." in k for k in keys):
        return "mal"
    if not any(".attention." in k for k in keys):
        return "lmm"
    return "mag"


def _clean(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    return {k.removeprefix("_orig_mod.").removeprefix("module."): v for k, v in sd.items()}


def rng_state() -> dict[str, Any]:
    st = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        st["cuda"] = torch.cuda.get_rng_state_all()
    return st


def set_rng_state(st: dict[str, Any]) -> None:
    random.setstate(st["python"])
    np.random.set_state(st["numpy"])
    torch.set_rng_state(st["torch"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(st["cuda"])


def save_checkpoint(path: str, model: torch.nn.Module, optimizer=None, scheduler=None, *, global_step: int = 0,
                    epoch: int = 0, best_val_loss: float = float("inf"), model_type: str | None = None,
                    tokenizer_name: str | None = None, data_position: int | None = None,
                    train_config: dict | None = None, dtype: torch.dtype | None = None,
                    extra: dict | None = None, state_dict: dict | None = None) -> str:
    """Write a reference-loadable checkpoint (plus resume state) to ``path``
    (``state_dict``: the model's values when ``model.state_dict()`` does not
    hold them, e.g. parameters sharded over ranks)."""
    cfg: TitansConfig = model.config
    src = model.state_dict() if state_dict is None else state_dict
    sd = {k: (v.to(dtype) if dtype is not None and v.is_floating_point() else v).detach().cpu()
          for k, v in src.items()}
    ckpt = {
        "model_state_dict": sd,
        "optimizer_state_dict": optimizer.state_dict() if optimizer is not None else None,
        "scheduler_state_dict": scheduler.state_dict() if scheduler is not None else None,
        "scaler_state_dict": None,
        "global_step": global_step,
        "epoch": epoch,
        "best_val_loss": best_val_loss,
        "config": cfg.to_dict(reference_only=True),
        "titans_b200_config": cfg.to_dict(),
        "model_type": model_type or getattr(model, "model_type", infer_model_type(sd)),
        "rng_state": rng_state(),
        "data_position": data_position,
        "train_config": train_config,
    }
    if tokenizer_name is not None:
        ckpt["tokenizer_name"] = tokenizer_name
    if extra:
        ckpt.update(extra)
    _atomic_save(ckpt, path)
    return path


def _atomic_save(obj, path: str) -> None:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)  # never leave a truncated checkpoint behind


def shard_path(path: str, rank: int, world: int) -> str:
    """File holding rank ``rank``'s optimizer shard of checkpoint ``path``."""
    return f"{path}.optim.rank{rank}-of-{world}"


def _barrier(group=None) -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier(group=group)


def save_training_checkpoint(path: str, trainer, *, rank: int = 0, world: int = 1, group=None, **meta) -> str:
    """Checkpoint of a (possibly data-parallel) training run; EVERY rank calls it.

    Parameters still sharded are gathered first.  An optimizer whose state is
    sharded over the ranks (``shard_state``) writes one file per rank
    (:func:`shard_path`) and rank 0 writes the reference-loadable model file
    with ``optimizer_shards = world``; otherwise rank 0 writes everything.  A
    host barrier at the end keeps every rank out of the next step until all
    files are on disk (the fused data-parallel step's device barriers have a
    time budget, and a long write on rank 0 must not run it out)."""
    opt = trainer.optimizer
    full = getattr(opt, "full_model_state_dict", None)
    model_sd = None
    if full is not None:  # every rank takes part in the gathers of sharded units
        model_sd = full(trainer.model)
    else:
        mat = getattr(opt, "materialize", None)
        if mat is not None:
            mat()
    sharded = world > 1 and getattr(opt, "shard_state", False)
    if sharded:
        sd = {k: (v.detach().cpu() if isinstance(v, torch.Tensor) else v) for k, v in opt.state_dict().items()}
        _atomic_save(sd, shard_path(path, rank, world))
    if rank == 0:
        save_checkpoint(path, trainer.model, None if sharded else opt, trainer.scheduler,
                        extra={"optimizer_shards": world if sharded else 0}, state_dict=model_sd, **meta)
    _barrier(group)
    return path


def load_training_checkpoint(path: str, trainer, *, rank: int = 0, world: int = 1, restore_rng: bool = True) -> dict:
    """Restore :func:`save_training_checkpoint` output on every rank (weights,
    scheduler, RNG, and this rank's optimizer shard or the full optimizer)."""
    ckpt = load_checkpoint(path, trainer.model, None, trainer.scheduler, restore_rng=restore_rng)
    opt = trainer.optimizer
    shards = int(ckpt.get("optimizer_shards") or 0)
    if shards:
        if shards != world:
            raise ValueError(f"{path}: optimizer saved over {shards} ranks, resuming on {world}")
        sd = torch.load(shard_path(path, rank, world), map_location="cpu", weights_only=False)
        opt.load_state_dict(sd)
    elif ckpt.get("optimizer_state_dict") is not None:
        opt.load_state_dict(ckpt["optimizer_state_dict"])
    return ckpt


def load_model(path: str, device=None, dtype: torch.dtype | None = None, **config_overrides):
    """Build the model a checkpoint describes and load its weights; returns (model, ckpt)."""
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    if not isinstance(ckpt, dict) or "model_state_dict" not in ckpt:
        raise ValueError(f"{path}: not a Titans checkpoint (no model_state_dict)")
    sd = _clean(ckpt["model_state_dict"])
    raw = ckpt.get("titans_b200_config") or ckpt.get("config") or {}
    cfg = TitansConfig.from_dict({**raw, **config_overrides})
    kind = ckpt.get("model_type") or infer_model_type(sd)
    model = MODEL_CLASSES[kind](cfg)
    model.load_state_dict(sd, strict=True)
    model = model.to(device=device, dtype=dtype) if (device or dtype) else model
    return model, ckpt


def load_checkpoint(path: str, model: torch.nn.Module, optimizer=None, scheduler=None,
                    restore_rng: bool = True, map_location="cpu") -> dict:
    """Restore weights (and optimizer / scheduler / RNG when given); returns the checkpoint dict."""
    ckpt = torch.load(path, map_location=map_location, weights_only=False)
    sd = _clean(ckpt["model_state_dict"])
    with torch.no_grad():
        model.load_state_dict({k: v.to(model.state_dict()[k].dtype) for k, v in sd.items()}, strict=True)
    if optimizer is not None and ckpt.get("optimizer_state_dict") is not None:
        optimizer.load_state_dict(ckpt["optimizer_state_dict"])
    if scheduler is not None and ckpt.get("scheduler_state_dict") is not None:
        scheduler.load_state_dict(ckpt["scheduler_state_dict"])
    if restore_rng and ckpt.get("rng_state") is not None:
        set_rng_state(ckpt["rng_state"])
    return ckpt
