"""BABILong-style needle QA (`scripts/benchmark_babilong.py:125-558`).

Examples come from the Hugging Face ``RMT-team/babilong`` dataset when it is in
the local cache, else from a synthetic generator with the same shape (filler
text with the supporting facts planted at random depths, then the question),
which is also the reference's fallback.  Each example is prefilled chunk by
chunk with carried memory states, then the answer is decoded greedily; the
score is exact match of the first answer word.
"""

from __future__ import annotations

import argparse
import json
import random

import torch

from ..inference.generate import generate, prefill
from ..utils.checkpoint import load_model
from ..utils.tokenizer import load_tokenizer

CONTEXTS = {"0k": 0, "1k": 1024, "2k": 2048, "4k": 4096, "8k": 8192, "16k": 16384, "32k": 32768,
            "64k": 65536, "128k": 131072}
NAMES = ["Mary", "John", "Sandra", "Daniel"]
PLACES = ["kitchen", "garden", "office", "bathroom", "hallway", "bedroom"]


def synthetic_examples(n: int, context_chars: int, seed: int = 0) -> list[dict]:
    rng = random.Random(seed)
    filler = "The grass is green. The sky is blue. Birds sing in the morning. "
    out = []
    for _ in range(n):
        who, where = rng.choice(NAMES), rng.choice(PLACES)
        fact = f" {who} went to the {where}. "
        body = (filler * (context_chars // len(filler) + 1))[:context_chars]
        cut = rng.randint(0, len(body))
        out.append({"input": body[:cut] + fact + body[cut:], "question": f"Where is {who}?", "target": where})
    return out


def load_examples(task: str, context: str, n: int) -> list[dict]:
    try:
        from datasets import load_dataset

        ds = load_dataset("RMT-team/babilong", context, split=task)
        return [dict(input=e["input"], question=e["question"], target=e["target"]) for e in ds.select(range(n))]
    except Exception:
        return synthetic_examples(n, CONTEXTS[context])


@torch.no_grad()
def answer(model, tok, ex: dict, max_new_tokens: int = 8) -> str:
    dev = next(model.parameters()).device
    ids = torch.tensor([tok.encode(ex["input"] + " " + ex["question"] + " Answer:", add_special_tokens=False)],
                       dtype=torch.long, device=dev)
    cs = model.config.chunk_size
    head, tail = ids[:, :max(0, ids.shape[1] - cs)], ids[:, -cs:]
    states = prefill(model, head)[1] if head.shape[1] else None
    out, _ = generate(model, tail, max_new_tokens, greedy=True, states=states)
    return tok.decode(out[0, tail.shape[1]:].tolist())


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="BABILong QA accuracy of a Titans checkpoint")
    a = p.add_argument
    a("--checkpoint", required=True)
    a("--tokenizer", default=None)
    a("--task", default="qa1")
    a("--context-length", choices=sorted(CONTEXTS), default="0k")
    a("--max-examples", type=int, default=50)
    a("--output", default=None)
    a("--device", default=None)
    args = p.parse_args(argv)
    dev = torch.device(args.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model, ckpt = load_model(args.checkpoint, device=dev, dtype=torch.bfloat16 if dev.type == "cuda" else None)
    model.eval()
    tok = load_tokenizer(args.tokenizer or ckpt.get("tokenizer_name"), model.config.vocab_size)
    tasks = [f"qa{i}" for i in range(1, 11)] if args.task == "all" else [args.task]
    results = {}
    for t in tasks:
        exs = load_examples(t, args.context_length, args.max_examples)
        correct = sum(int(ex["target"].lower() in answer(model, tok, ex).lower().split()[:3]) for ex in exs)
        results[t] = correct / max(len(exs), 1)
    print(json.dumps(results))
    if args.output:
        with open(args.output, "w", encoding="utf-8") as f:
            json.dump({"results": results, "context": args.context_length}, f, indent=2)


if __name__ == "__main__":
    main()
