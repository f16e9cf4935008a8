"""Perplexity evaluation (`scripts/eval_perplexity.py:167-468`).

Two modes, as in the reference:
* strided sliding window (``--max-length``, ``--stride``): each window is an
  independent forward; only the tokens not scored by the previous window count;
* ``--use-memory``: the text is fed in ``--chunk-size`` slices with the memory
  states carried between slices (how Titans scales to long inputs).

Text comes from ``--data`` (a local file) or a local Hugging Face dataset
(``--dataset`` name resolved from the local cache; no network).
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from ..ops.loss import cross_entropy
from ..utils.checkpoint import load_model
from ..utils.tokenizer import load_tokenizer

DATASETS = {"wikitext-2": ("wikitext", "wikitext-2-raw-v1"), "wikitext-103": ("wikitext", "wikitext-103-raw-v1"),
            "pg19": ("pg19", None), "lambada": ("lambada", None)}


@torch.no_grad()
def perplexity_sliding(model, ids: torch.Tensor, max_length: int = 4096, stride: int = 512) -> dict:
    nll, count, prev_end = 0.0, 0, 0
    T = ids.shape[1]
    for begin in range(0, T, stride):
        end = min(begin + max_length, T)
        trg = end - prev_end
        x = ids[:, begin:end]
        y = x.clone()
        y[:, :-trg] = -100
        logits, _ = model(x)
        lab = y[:, 1:]
        n = int((lab != -100).sum())
        if n:
            nll += float(cross_entropy(logits[:, :-1], lab)) * n
            count += n
        prev_end = end
        if end == T:
            break
    avg = nll / max(count, 1)
    return {"loss": avg, "perplexity": math.exp(min(avg, 50)), "tokens": count}


@torch.no_grad()
def perplexity_with_memory(model, ids: torch.Tensor, chunk_size: int = 512) -> dict:
    nll, count, states = 0.0, 0, None
    T = ids.shape[1]
    for s in range(0, T - 1, chunk_size):
        x = ids[:, s:min(s + chunk_size, T - 1)]
        y = ids[:, s + 1:s + 1 + x.shape[1]]
        logits, states = model(x, states=states)
        n = y.numel()
        nll += float(cross_entropy(logits, y)) * n
        count += n
    avg = nll / max(count, 1)
    return {"loss": avg, "perplexity": math.exp(min(avg, 50)), "tokens": count}


def load_text(args) -> str:
    if args.data:
        with open(args.data, encoding="utf-8") as f:
            return f.read()
    from datasets import load_dataset

    name, sub = DATASETS[args.dataset]
    ds = load_dataset(name, sub, split="test")
    return "\n\n".join(ds["text"])


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Perplexity of a Titans checkpoint")
    a = p.add_argument
    a("--checkpoint", required=True)
    a("--tokenizer", default=None)
    a("--dataset", choices=sorted(DATASETS), default="wikitext-2")
    a("--data", default=None)
    a("--max-length", type=int, default=4096)
    a("--stride", type=int, default=512)
    a("--use-memory", action="store_true")
    a("--chunk-size", type=int, default=512)
    a("--max-tokens", type=int, default=0, help="evaluate only the first N tokens (0 = all)")
    a("--output", default=None)
    a("--device", default=None)
    args = p.parse_args(argv)
    dev = torch.device(args.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model, ckpt = load_model(args.checkpoint, device=dev, dtype=torch.bfloat16 if dev.type == "cuda" else None)
    model.eval()
    tok = load_tokenizer(args.tokenizer or ckpt.get("tokenizer_name"), model.config.vocab_size)
    ids = torch.tensor([tok.encode(load_text(args), add_special_tokens=False)], dtype=torch.long, device=dev)
    if args.max_tokens:
        ids = ids[:, :args.max_tokens]
    res = (perplexity_with_memory(model, ids, args.chunk_size) if args.use_memory
           else perplexity_sliding(model, ids, args.max_length, args.stride))
    print(json.dumps(res))
    if args.output:
        with open(args.output, "w", encoding="utf-8") as f:
            json.dump({**res, "checkpoint": args.checkpoint, "mode": "memory" if args.use_memory else "sliding"},
                      f, indent=2)


if __name__ == "__main__":
    main()
