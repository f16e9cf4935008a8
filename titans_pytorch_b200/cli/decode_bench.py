"""Decode throughput: the reference's recurrence vs incremental decoding (bf16, int8 weights).

    python -m titans_pytorch_b200.cli.decode_bench --batch 1 --prompt 512 --new 64

Three decoders on the same random-init model (default: the TitansMAG ~170M
training architecture, bf16):

* ``recurrence``: ``generate()`` -- every new token re-runs the model on the
  last ``chunk_size`` tokens with carried memory states (the reference's
  decoding, `scripts/inference.py:321-423`);
* ``streaming``: :class:`~titans_pytorch_b200.inference.decode.StreamingDecoder`
  -- one token per step over a sliding-window KV ring and the carried memory,
  the step captured once in a CUDA graph and replayed (``--no-graph``: eager);
* ``streaming_int8``: the same with int8 weights (``ops.quant``).

Timed with CUDA events around the decode loop after a prompt prefill and
one warm-up token; one JSON line per decoder (tokens/s over batch x new
tokens, weight bytes).
"""

from __future__ import annotations

import argparse
import copy
import json

import torch


def _weight_bytes(model) -> int:
    from ..ops.quant import Int8Weight

    total, seen = 0, set()
    for mod in model.modules():
        for name, p in list(mod._parameters.items()) + [("weight", getattr(mod, "weight", None))]:
            if p is None or id(p) in seen or not isinstance(p, torch.Tensor):
                continue
            seen.add(id(p))
            total += p.nbytes_stored() if isinstance(p, Int8Weight) else p.numel() * p.element_size()
    return total


def main(argv=None) -> None:
    from .. import TitansConfig, create_model
    from ..inference.decode import StreamingDecoder
    from ..inference.generate import generate
    from ..ops.quant import quantize_model_int8

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="mag", choices=["mag", "mal", "lmm"])
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--window", type=int, default=512)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=256)
    ap.add_argument("--new", type=int, default=32)
    ap.add_argument("--which", default="recurrence,streaming,streaming_int8")
    ap.add_argument("--no-graph", action="store_true", help="streaming decoders: eager steps (no CUDA graph)")
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    cfg = TitansConfig(vocab_size=a.vocab, dim=a.dim, num_layers=a.layers, num_heads=a.heads,
                       window_size=a.window, chunk_size=a.chunk, num_memory_layers=2, num_persistent_tokens=4,
                       max_seq_len=max(4096, a.prompt + a.new), dropout=0.0)
    base = create_model(a.model, cfg).cuda().to(torch.bfloat16).eval()
    ids = torch.randint(0, a.vocab, (a.batch, a.prompt), device="cuda")
    nxt = torch.randint(0, a.vocab, (a.batch, a.new), device="cuda")
    for which in a.which.split(","):
        model = copy.deepcopy(base)
        if which == "streaming_int8":
            quantize_model_int8(model)
            torch.cuda.empty_cache()
        wbytes = _weight_bytes(model)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.no_grad():
            if which == "recurrence":
                _, st = model(ids[:, -cfg.chunk_size:])
                generate(model, ids, 1, greedy=True, states=st)  # warm-up
                torch.cuda.synchronize()
                s.record()
                generate(model, ids, a.new, greedy=True, states=st)
                e.record()
            else:
                dec = StreamingDecoder(model, batch=a.batch, graph=not a.no_graph)
                dec.prefill(ids)
                dec.step(nxt[:, :1])  # warm-up
                torch.cuda.synchronize()
                s.record()
                for t in range(a.new):
                    dec.step(nxt[:, t:t + 1])
                e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        print(json.dumps({"decoder": which, "model": a.model, "batch": a.batch, "new_tokens": a.new,
                          "ms_per_token": round(ms / a.new, 3), "tokens_per_s": round(a.batch * a.new / ms * 1e3, 1),
                          "weight_gib": round(wbytes / 2 ** 30, 3)}), flush=True)


if __name__ == "__main__":
    main()
