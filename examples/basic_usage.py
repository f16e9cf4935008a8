"""Tour of the public API (the reference's `examples/basic_usage.py` topics).

    python examples/basic_usage.py            # CPU, tiny sizes
    python examples/basic_usage.py --device cuda

Covers: configuration, the four model variants, a forward pass with carried
memory states, one training step through the Trainer (fused AdamW, clipping,
cosine schedule), generation, and a checkpoint round trip in the reference's
format.
"""

from __future__ import annotations

import argparse
import os
import tempfile

import torch

import titans_pytorch_b200 as titans


def tiny_config(**kw) -> titans.TitansConfig:
    base = dict(dim=64, num_heads=4, num_layers=2, vocab_size=256, chunk_size=32, window_size=16,
                num_persistent_tokens=4, num_memory_layers=2, dropout=0.0, max_seq_len=256)
    base.update(kw)
    return titans.TitansConfig(**base)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--device", default="cpu")
    args = p.parse_args(argv)
    dev = torch.device(args.device)
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    torch.manual_seed(0)

    cfg = tiny_config()
    print(f"config: dim={cfg.dim} heads={cfg.num_heads} head_dim={cfg.head_dim} ffn_dim={cfg.ffn_dim} "
          f"memory_hidden_dim={cfg.memory_hidden_dim}")

    # 1. the four variants share one forward signature: (logits, states)
    ids = torch.randint(0, cfg.vocab_size, (2, 64), device=dev)
    for kind in ("mac", "mag", "mal", "lmm"):
        model = titans.create_model(kind, cfg).to(dev, dtype)
        logits, states = model(ids)
        n = sum(p.numel() for p in model.parameters())
        print(f"{kind}: params={n:,} logits={tuple(logits.shape)} memory states={len(states)}")

    # 2. memory persistence: feed a sequence in two calls, carrying the states
    model = titans.TitansMAG(cfg).to(dev, dtype).eval()
    with torch.no_grad():
        _, st = model(ids[:, :32])
        second, st = model(ids[:, 32:], states=st)
    print(f"second half with carried memory: logits {tuple(second.shape)}")

    # 3. one training step (returns the loss on the device)
    trainer = titans.Trainer(titans.TitansMAG(cfg), titans.TrainStepConfig(lr=3e-4, dtype=dtype), device=dev)
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    loss = trainer.train_step(batch)
    print(f"train step: loss={float(loss):.4f}")

    # 4. generation (greedy, then sampled)
    prompt = ids[:1, :8]
    out, _ = titans.generate(trainer.model.eval(), prompt, max_new_tokens=8, greedy=True)
    print(f"generated ids: {out[0, 8:].tolist()}")

    # 5. checkpoint round trip (loadable by the reference's loaders too)
    with tempfile.TemporaryDirectory() as d:
        path = titans.save_checkpoint(os.path.join(d, "ckpt.pt"), trainer.model, trainer.optimizer,
                                      global_step=trainer.global_step)
        loaded, ck = titans.load_model(path, device=dev, dtype=dtype)
        print(f"checkpoint: model_type={ck['model_type']} step={ck['global_step']} "
              f"params equal={all(torch.equal(a, b) for a, b in zip(trainer.model.state_dict().values(), loaded.state_dict().values()))}")


if __name__ == "__main__":
    main()
