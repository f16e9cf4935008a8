"""Long inputs with the neural memory (the reference's `examples/long_sequence.py` topics).

    python examples/long_sequence.py                     # CPU, tiny sizes
    python examples/long_sequence.py --device cuda --tokens 131072 --dim 1024 --layers 24

Three demos:
* chunked processing: a long sequence is fed in `chunk` slices with the memory
  states carried between calls, so cost grows linearly with length;
* streaming: tokens arrive in small pieces and the memory keeps the context;
* persistence: the memory states are saved, reloaded and used to continue.
"""

from __future__ import annotations

import argparse
import time

import torch

import titans_pytorch_b200 as titans
from titans_pytorch_b200.inference.generate import prefill


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--device", default="cpu")
    p.add_argument("--model", default="mac", choices=["mac", "mag", "mal", "lmm"])
    p.add_argument("--tokens", type=int, default=1024)
    p.add_argument("--chunk", type=int, default=128)
    p.add_argument("--dim", type=int, default=64)
    p.add_argument("--layers", type=int, default=2)
    args = p.parse_args(argv)
    dev = torch.device(args.device)
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    torch.manual_seed(0)
    cfg = titans.TitansConfig(dim=args.dim, num_heads=max(1, args.dim // 64) if args.dim >= 64 else 2,
                              num_layers=args.layers, vocab_size=256, chunk_size=args.chunk,
                              window_size=args.chunk, num_persistent_tokens=4, dropout=0.0,
                              max_seq_len=max(args.tokens, 1024))
    model = titans.create_model(args.model, cfg).to(dev, dtype).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, args.tokens), device=dev)

    # chunked processing with carried memory
    t0 = time.perf_counter()
    last, states = prefill(model, ids, chunk=args.chunk)
    if dev.type == "cuda":
        torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    print(f"chunked prefill: {args.tokens} tokens in {dt:.3f} s ({args.tokens / dt:,.0f} tok/s), "
          f"last logits {tuple(last.shape)}")

    # streaming: 16-token pieces
    st = None
    with torch.no_grad():
        for a in range(0, min(args.tokens, 256), 16):
            _, st = model(ids[:, a:a + 16], states=st)
    print(f"streaming: {min(args.tokens, 256) // 16} pieces, memory layers carried: {len(st)}")

    # persistence: save the states, reload, continue
    saved = [s.detach() for s in states]
    buf = {"weights": [[w.cpu() for w in s.weights] for s in saved],
           "momentum": [[m.cpu() for m in s.momentum] for s in saved]}
    restored = [titans.MemoryState([w.to(dev) for w in ws], [m.to(dev) for m in ms])
                for ws, ms in zip(buf["weights"], buf["momentum"])]
    with torch.no_grad():
        a, _ = model(ids[:, -args.chunk:], states=saved)
        b, _ = model(ids[:, -args.chunk:], states=restored)
    print(f"persistence: continuation identical after reload = {torch.equal(a, b)}")


if __name__ == "__main__":
    main()
