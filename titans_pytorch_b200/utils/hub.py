"""Hugging Face Hub layout: ``pytorch_model.bin`` + ``config.json`` + model card.

Same layout as the reference (`src/titans/hub.py:67-239`): ``config.json``
holds ``{"model_type", "titans_config", "tokenizer_name"}``.  ``push_to_hub``
writes the layout into a local directory (this is also the staging step of an
upload) and uploads it with ``huggingface_hub`` only when ``upload=True`` and
the package is available; ``load_from_hub`` reads a local directory or, if
that does not exist, tries ``huggingface_hub.snapshot_download``.
"""

from __future__ import annotations

import json
import os

import torch

from ..config import TitansConfig
from ..models.titans import MODEL_CLASSES
from .checkpoint import infer_model_type, load_model


def _estimate_params(config: dict, model_type: str) -> int:
    """Parameter count of a config without building the model (meta device)."""
    with torch.device("meta"):
        m = MODEL_CLASSES[model_type](TitansConfig.from_dict(config))
    return sum(p.numel() for p in m.parameters())


def _model_card(model_type: str, cfg: dict, n_params: int, tokenizer_name: str | None) -> str:
    lines = [f"# Titans-{model_type.upper()}", "",
             f"Titans ({model_type.upper()}) language model, {n_params / 1e6:.1f}M parameters.", "",
             "| field | value |", "|---|---|"]
    lines += [f"| {k} | {v} |" for k, v in sorted(cfg.items())]
    if tokenizer_name:
        lines += ["", f"Tokenizer: `{tokenizer_name}`"]
    return "\n".join(lines) + "\n"


def save_pretrained(model: torch.nn.Module, directory: str, tokenizer_name: str | None = None) -> str:
    os.makedirs(directory, exist_ok=True)
    kind = getattr(model, "model_type", None) or infer_model_type(model.state_dict())
    cfg = model.config.to_dict(reference_only=True)
    torch.save({k: v.detach().cpu() for k, v in model.state_dict().items()},
               os.path.join(directory, "pytorch_model.bin"))
    with open(os.path.join(directory, "config.json"), "w", encoding="utf-8") as f:
        json.dump({"model_type": kind, "titans_config": cfg, "tokenizer_name": tokenizer_name}, f, indent=2)
    n = sum(p.numel() for p in model.parameters())
    with open(os.path.join(directory, "README.md"), "w", encoding="utf-8") as f:
        f.write(_model_card(kind, cfg, n, tokenizer_name))
    return directory


def push_to_hub(model: torch.nn.Module, repo_id: str, tokenizer_name: str | None = None,
                local_dir: str | None = None, upload: bool = False, private: bool = False,
                token: str | None = None) -> str:
    d = save_pretrained(model, local_dir or repo_id.replace("/", "__"), tokenizer_name)
    if upload:
        from huggingface_hub import HfApi

        api = HfApi(token=token)
        api.create_repo(repo_id, private=private, exist_ok=True)
        api.upload_folder(folder_path=d, repo_id=repo_id)
    return d


def load_from_hub(repo_or_dir: str, device=None, dtype: torch.dtype | None = None, **overrides):
    d = repo_or_dir
    if not os.path.isdir(d):
        from huggingface_hub import snapshot_download

        d = snapshot_download(repo_or_dir)
    with open(os.path.join(d, "config.json"), encoding="utf-8") as f:
        meta = json.load(f)
    cfg = TitansConfig.from_dict({**meta["titans_config"], **overrides})
    model = MODEL_CLASSES[meta["model_type"]](cfg)
    model.load_state_dict(torch.load(os.path.join(d, "pytorch_model.bin"), map_location="cpu"), strict=True)
    return model.to(device=device, dtype=dtype) if (device or dtype) else model


def convert_checkpoint_to_hub_format(checkpoint_path: str, output_dir: str,
                                     tokenizer_name: str | None = None) -> str:
    model, ckpt = load_model(checkpoint_path)
    return save_pretrained(model, output_dir, tokenizer_name or ckpt.get("tokenizer_name"))
