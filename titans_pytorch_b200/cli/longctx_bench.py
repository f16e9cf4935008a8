"""Long-context MAC inference: prefill and decode throughput on one GPU.

    python -m titans_pytorch_b200.cli.longctx_bench                     # this framework
    python -m titans_pytorch_b200.cli.longctx_bench --impl reference    # the reference package

Model: TitansMAC with the ~400M training architecture (vocab 32000, dim 1024,
24 layers, 16 heads, segment 512, 16 persistent tokens, L_M=2), random bf16
weights (std 0.02).  Prompt: ``--prefill`` (default 131072) uniform filler ids
over [0, 32000), with an 8-token key and an 8-token value planted at a random
offset and the key repeated at the end.

* Prefill: the prompt minus its last segment goes through the model in
  ``--piece``-token calls with the memory states carried (the model segments
  each call internally), at batch ``--prefill-batch``.
* Decode: ``--new-tokens`` greedy tokens at batch 1 and 16, each produced the
  reference's way (`scripts/inference.py:321-423`): the last segment is re-run
  with the carried states.

This framework replays both phases from CUDA graphs (``GraphedForward``:
one graph per input shape with the memory states chained in place; the first
prefill piece runs eagerly to seed the states, capture is outside the timed
phases); ``--no-graphs`` runs them eagerly.  The reference arm runs its
model's own forward eagerly.

Timing: CUDA events around each phase after one untimed warm-up decode step.
One JSON line: prefill tokens/s and decode tokens/s (new tokens x batch / s).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

FIELDS = dict(vocab_size=32000, dim=1024, num_layers=24, num_heads=16, chunk_size=512, window_size=512,
              num_memory_layers=2, memory_hidden_mult=4.0, ffn_mult=4.0, num_persistent_tokens=16,
              conv_kernel_size=4, use_conv=True, use_rope=True, dropout=0.0, max_seq_len=1 << 18, init_std=0.02)


def make_prompt(B: int, T: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, FIELDS["vocab_size"], (B, T), generator=g)
    key = torch.randint(0, FIELDS["vocab_size"], (B, 8), generator=g)
    val = torch.randint(0, FIELDS["vocab_size"], (B, 8), generator=g)
    off = int(torch.randint(0, T - 32, (1,), generator=g))
    ids[:, off:off + 8] = key
    ids[:, off + 8:off + 16] = val
    ids[:, T - 8:] = key
    return ids


def build(impl: str, device):
    torch.manual_seed(0)
    if impl == "reference":
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        sys.path.insert(0, os.path.join(root, "baseline", "_ref"))
        import titans

        model = titans.TitansMAC(titans.TitansConfig(**FIELDS))
    else:
        import titans_pytorch_b200 as titans

        model = titans.TitansMAC(titans.TitansConfig(**FIELDS))
    return model.to(device=device, dtype=torch.bfloat16).eval()


@torch.no_grad()
def prefill(model, ids, piece):
    states = None
    for s in range(0, ids.shape[1], piece):
        _, states = model(ids[:, s:s + piece], states=states)
    return states


@torch.no_grad()
def decode(model, ctx, states, n, seg):
    gen = ctx
    for _ in range(n):
        logits, states = model(gen[:, -seg:], states=states)
        gen = torch.cat([gen, logits[:, -1].argmax(-1, keepdim=True)], 1)
    return gen, states


def timed(fn):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    out = fn()
    e.record()
    torch.cuda.synchronize()
    return out, s.elapsed_time(e)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--prefill", type=int, default=131072)
    p.add_argument("--prefill-batch", type=int, default=1)
    p.add_argument("--piece", type=int, default=8192)
    p.add_argument("--new-tokens", type=int, default=16)
    p.add_argument("--no-graphs", action="store_true")
    a = p.parse_args(argv)
    graphs = a.impl == "ours" and not a.no_graphs
    dev = torch.device("cuda")
    model = build(a.impl, dev)
    seg = FIELDS["chunk_size"]
    out = {"bench": "mac_long_context_inference", "impl": a.impl, "prefill_tokens": a.prefill,
           "model": "TitansMAC ~400M (dim 1024, 24 layers, 16 heads, segment 512, 16 persistent, L_M=2)"}
    ids = make_prompt(max(16, a.prefill_batch), a.prefill).to(dev)
    head, tail = ids[:, :-seg], ids[:, -seg:]
    # warm-up: one short prefill and one decode step
    st = prefill(model, head[:1, :seg * 2], a.piece)
    decode(model, tail[:1], st, 1, seg)
    torch.cuda.synchronize()
    B = a.prefill_batch
    out["cuda_graphs"] = graphs
    if graphs:
        from ..inference.generate import GraphedForward

        # the first piece runs eagerly (it seeds the state chain), the rest are replays
        first, ms0 = timed(lambda: prefill(model, head[:B, :a.piece], a.piece))
        runner = GraphedForward(model, B, a.piece, first)
        torch.cuda.synchronize()

        full = head.shape[1] // a.piece * a.piece

        def graphed_prefill():
            for s0 in range(a.piece, full, a.piece):
                runner(head[:B, s0:s0 + a.piece])
            if full == head.shape[1]:
                return runner.states
            with torch.no_grad():  # the shorter last piece runs eagerly
                return model(head[:B, full:], states=runner.states)[1]

        st, ms = timed(graphed_prefill)
        ms += ms0
    else:
        st, ms = timed(lambda: prefill(model, head[:B], a.piece))
    out["prefill"] = {"batch": B, "ms": round(ms, 1), "tokens_per_s": B * head.shape[1] / ms * 1e3}
    # reference-semantics memory states are shared by the batch, so the
    # prefilled states serve every decode batch size
    for bd in (1, 16):
        if graphs:
            step = GraphedForward(model, bd, seg, st)
            torch.cuda.synchronize()

            def graphed_decode():
                step.load_states(st)
                gen = tail[:bd]
                for _ in range(a.new_tokens):
                    logits, _ = step(gen[:, -seg:])
                    gen = torch.cat([gen, logits[:, -1].argmax(-1, keepdim=True)], 1)
                return gen

            _, ms = timed(graphed_decode)
        else:
            (_, _), ms = timed(lambda: decode(model, tail[:bd], st, a.new_tokens, seg))
        out[f"decode_b{bd}"] = {"new_tokens": a.new_tokens, "ms": round(ms, 1),
                                "tokens_per_s": bd * a.new_tokens / ms * 1e3}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
