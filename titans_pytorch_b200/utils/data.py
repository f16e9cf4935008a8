"""Datasets and host->device prefetching.

Datasets mirror the reference trainer's (`scripts/pretrain.py:182-373`):
``SyntheticDataset`` (uniform ids, seeded), ``TextFileDataset`` (tokenizer over
a text file), ``CharLevelDataset``, ``LocalHFDataset`` (pre-tokenized Arrow
dataset from ``save_to_disk``, memory-mapped) and ``StreamingDataset``
(Hugging Face streaming with per-worker sharding).  Every item is
``{"input_ids": x[:-1], "labels": x[1:]}``.

``CUDAPrefetcher`` (`src/titans/cuda_optimizations.py:445-492`) copies the next
batch from pinned host memory on a side stream while the current step runs and
hands it over with a stream event, so the H2D copy overlaps compute.
"""

from __future__ import annotations

import torch
from torch.utils.data import Dataset, IterableDataset, get_worker_info


class SyntheticDataset(Dataset):
    def __init__(self, vocab_size: int, seq_len: int, num_samples: int, seed: int = 42) -> None:
        g = torch.Generator().manual_seed(seed)
        self.data = torch.randint(0, vocab_size, (num_samples, seq_len + 1), generator=g)

    def __len__(self) -> int:
        return self.data.shape[0]

    def __getitem__(self, i):
        return {"input_ids": self.data[i, :-1], "labels": self.data[i, 1:]}


class _TokenStream(Dataset):
    def __init__(self, tokens: torch.Tensor, seq_len: int) -> None:
        self.tokens = tokens
        self.seq_len = seq_len

    def __len__(self) -> int:
        return max(0, self.tokens.numel() - self.seq_len)

    def __getitem__(self, i):
        return {"input_ids": self.tokens[i:i + self.seq_len], "labels": self.tokens[i + 1:i + self.seq_len + 1]}


class TextFileDataset(_TokenStream):
    def __init__(self, path: str, tokenizer, seq_len: int) -> None:
        with open(path, encoding="utf-8") as f:
            text = f.read()
        super().__init__(torch.tensor(tokenizer.encode(text, add_special_tokens=False), dtype=torch.long), seq_len)


class CharLevelDataset(_TokenStream):
    def __init__(self, path: str, vocab_size: int, seq_len: int) -> None:
        with open(path, encoding="utf-8") as f:
            text = f.read()
        table = {c: i % vocab_size for i, c in enumerate(sorted(set(text)))}
        self.char_to_idx = table
        super().__init__(torch.tensor([table.get(c, 0) for c in text], dtype=torch.long), seq_len)


class LocalHFDataset(Dataset):
    """Pre-tokenized dataset written by ``pretokenize`` (``input_ids`` of length seq_len + 1)."""

    def __init__(self, path: str, seq_len: int | None = None) -> None:
        from datasets import load_from_disk

        self.dataset = load_from_disk(path)
        first = self.dataset[0]
        if "input_ids" not in first or not isinstance(first["input_ids"], (list, tuple)):
            raise ValueError("raw-text datasets are not supported: pre-tokenize them first")
        self.seq_len = seq_len

    def __len__(self) -> int:
        return len(self.dataset)

    def __getitem__(self, i):
        t = torch.tensor(self.dataset[i]["input_ids"], dtype=torch.long)
        return {"input_ids": t[:-1], "labels": t[1:]}


class StreamingDataset(IterableDataset):
    """Hugging Face streaming dataset, tokenized on the fly, each worker on its own shard."""

    def __init__(self, dataset_name: str, tokenizer, seq_len: int, subset: str | None = None,
                 split: str = "train", text_field: str = "text") -> None:
        self.dataset_name, self.subset, self.split = dataset_name, subset, split
        self.tokenizer, self.seq_len, self.text_field = tokenizer, seq_len, text_field

    def __iter__(self):
        from datasets import load_dataset

        ds = load_dataset(self.dataset_name, self.subset, split=self.split, streaming=True)
        info = get_worker_info()
        if info is not None and info.num_workers > 1:
            ds = ds.shard(num_shards=info.num_workers, index=info.id)
        buf: list[int] = []
        n = self.seq_len + 1
        for ex in ds:
            buf.extend(self.tokenizer.encode(ex[self.text_field], add_special_tokens=False))
            while len(buf) >= n:
                t = torch.tensor(buf[:n], dtype=torch.long)
                buf = buf[n:]  # no overlap between consecutive windows
                yield {"input_ids": t[:-1], "labels": t[1:]}


class CUDAPrefetcher:
    """Iterate a loader with the next batch's H2D copy overlapped on a side stream."""

    def __init__(self, loader, device) -> None:
        self.loader = loader
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None

    def __iter__(self):
        it = iter(self.loader)
        nxt = self._load(it)
        while nxt is not None:
            batch, ev = nxt
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
                for v in batch.values():
                    if isinstance(v, torch.Tensor):
                        v.record_stream(torch.cuda.current_stream(self.device))
            nxt = self._load(it)
            yield batch

    def _load(self, it):
        try:
            b = next(it)
        except StopIteration:
            return None
        if self.stream is None:
            return {k: v.to(self.device) for k, v in b.items()}, None
        with torch.cuda.stream(self.stream):
            out = {k: (v.pin_memory() if not v.is_pinned() else v).to(self.device, non_blocking=True)
                   for k, v in b.items()}
            ev = torch.cuda.Event()
            ev.record(self.stream)
        return out, ev
