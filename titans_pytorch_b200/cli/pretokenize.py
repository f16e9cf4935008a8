"""Pre-tokenize a text dataset into fixed windows (`scripts/pretokenize.py:42-175`).

Windows of ``seq_len + 1`` tokens with stride ``seq_len`` (consecutive windows
share one token, so every position is a target once), saved with
``save_to_disk`` for :class:`~titans_pytorch_b200.utils.data.LocalHFDataset`.
Input is a local text file (``--input``) or a dataset in the local Hugging Face
cache (``--dataset``).
"""

from __future__ import annotations

import argparse

from ..utils.tokenizer import load_tokenizer


def windows(tokens: list[int], seq_len: int) -> list[list[int]]:
    return [tokens[s:s + seq_len + 1] for s in range(0, len(tokens) - seq_len, seq_len)]


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Pre-tokenize text into training windows")
    a = p.add_argument
    a("--dataset", default=None)
    a("--subset", default=None)
    a("--split", default="train")
    a("--input", default=None, help="local text file")
    a("--tokenizer", default=None)
    a("--vocab-size", type=int, default=256, help="char-level tokenizer vocabulary when no tokenizer is given")
    a("--output", required=True)
    a("--seq-len", type=int, default=2048)
    a("--max-samples", type=int, default=0)
    args = p.parse_args(argv)
    from datasets import Dataset

    tok = load_tokenizer(args.tokenizer, args.vocab_size)
    if args.input:
        with open(args.input, encoding="utf-8") as f:
            texts = [f.read()]
    else:
        from datasets import load_dataset

        texts = load_dataset(args.dataset, args.subset, split=args.split)["text"]
    toks: list[int] = []
    for t in texts:
        toks.extend(tok.encode(t, add_special_tokens=False))
    rows = windows(toks, args.seq_len)
    if args.max_samples:
        rows = rows[:args.max_samples]
    Dataset.from_dict({"input_ids": rows}).save_to_disk(args.output)
    print(f"wrote {len(rows)} windows of {args.seq_len + 1} tokens to {args.output}")


if __name__ == "__main__":
    main()
