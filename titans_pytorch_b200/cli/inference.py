"""Text generation CLI (`scripts/inference.py:476-691` flags).

    python -m titans_pytorch_b200.cli.inference --checkpoint ckpt.pt --prompt "Once" --max-tokens 50
"""

from __future__ import annotations

import argparse
import sys

import torch

from ..inference.generate import generate, quantize_model_dynamic
from ..utils.checkpoint import load_model
from ..utils.tokenizer import load_tokenizer


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Generate text with a Titans checkpoint")
    a = p.add_argument
    a("--checkpoint", required=True)
    a("--tokenizer", default=None)
    a("--prompt", default="")
    a("--max-tokens", type=int, default=100)
    a("--temperature", type=float, default=1.0)
    a("--top-k", type=int, default=50)
    a("--top-p", type=float, default=0.9)
    a("--repetition-penalty", type=float, default=1.0)
    a("--interactive", action="store_true")
    a("--stream", action="store_true")
    a("--quantize", choices=["int8", "int4", "fp16"], default=None)
    a("--decoder", choices=["recurrence", "incremental"], default="recurrence",
      help="recurrence: re-run the last chunk per token (the reference's decoding); incremental: one "
           "token per step over a sliding-window KV cache with the memory state carried (MAG / MAL / LMM)")
    a("--device", default=None)
    a("--seed", type=int, default=0)
    return p


def run_prompt(model, tok, prompt: str, args, out=sys.stdout) -> str:
    dev = next(model.parameters()).device
    ids = tok.encode(prompt or " ", add_special_tokens=False) if hasattr(tok, "encode") else tok(prompt)
    x = torch.tensor([ids], dtype=torch.long, device=dev)
    kw = dict(temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
              repetition_penalty=args.repetition_penalty, eos_token_id=getattr(tok, "eos_token_id", None))
    if getattr(args, "decoder", "recurrence") == "incremental" and getattr(model, "model_type", "") != "mac":
        from ..inference.decode import generate_incremental

        ids_, _ = generate_incremental(model, x, args.max_tokens, **kw)
        text = tok.decode(ids_[0, x.shape[1]:].tolist())
        out.write(prompt + text + "\n")
        return text
    if getattr(args, "decoder", "recurrence") == "incremental":
        print("note: MAC decodes with the recurrence (no incremental decoder for it)", file=sys.stderr)
    if args.stream:
        text, n0 = "", x.shape[1]
        for ids_, _ in generate(model, x, args.max_tokens, stream=True, **kw):
            piece = tok.decode(ids_[0, n0:].tolist())
            out.write(piece[len(text):])
            out.flush()
            text = piece
        out.write("\n")
        return text
    ids_, _ = generate(model, x, args.max_tokens, **kw)
    text = tok.decode(ids_[0, x.shape[1]:].tolist())
    out.write(prompt + text + "\n")
    return text


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    torch.manual_seed(args.seed)
    device = torch.device(args.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    model, ckpt = load_model(args.checkpoint, device=device, dtype=dtype)
    model.eval()
    if args.quantize in ("int8", "int4"):
        quantize_model_dynamic(model, bits=8 if args.quantize == "int8" else 4)
    tok = load_tokenizer(args.tokenizer or ckpt.get("tokenizer_name"), model.config.vocab_size)
    if args.interactive:
        while True:
            try:
                prompt = input("> ")
            except EOFError:
                break
            if prompt.strip() in ("quit", "exit"):
                break
            run_prompt(model, tok, prompt, args)
    else:
        run_prompt(model, tok, args.prompt, args)


if __name__ == "__main__":
    main()
