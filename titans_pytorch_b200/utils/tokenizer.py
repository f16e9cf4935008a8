"""Tokenizer loading: a Hugging Face tokenizer when available (local files,
no network), else a character-level tokenizer like the reference's fallback
(`scripts/inference.py:61-107`)."""

from __future__ import annotations


class SimpleTokenizer:
    """Characters -> code points modulo the vocabulary."""

    def __init__(self, vocab_size: int = 256) -> None:
        self.vocab_size = vocab_size
        self.eos_token_id = None

    def encode(self, text: str, add_special_tokens: bool = False, return_tensors=None):
        ids = [ord(c) % self.vocab_size for c in text]
        if return_tensors == "pt":
            import torch

            return torch.tensor([ids], dtype=torch.long)
        return ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return "".join(chr(int(i)) for i in ids)

    def __call__(self, text: str, return_tensors=None):
        return {"input_ids": self.encode(text, return_tensors=return_tensors)}


def load_tokenizer(name: str | None, vocab_size: int = 256):
    if not name:
        return SimpleTokenizer(vocab_size)
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(name, local_files_only=True)
    except Exception:
        return SimpleTokenizer(vocab_size)
