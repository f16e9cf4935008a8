"""Training-throughput benchmark: TitansMAG ~170M (244.2M params), bf16, data parallel.

Workload (the reference's headline training config): vocab 32000, dim 768,
12 layers, 12 heads (head_dim 64), sliding window 512, memory depth L_M = 2
(hidden 4*dim), 4 persistent tokens, conv 4, RoPE, dropout 0; sequence 4096,
micro-batch 8 per GPU; synthetic token ids uniform over [0, 32000), random
init (std 0.02).  The memory update runs in the reference's semantics (one
update per forward over the whole sequence), so "memory chunk" does not apply.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

``--config`` (default ``mag170m``, the headline) also selects the larger
training workloads of the same metric: ``mac400m`` (TitansMAC, dim 1024, 24
layers, 16 heads, segment 512, 16 persistent tokens, L_M=2; sequence 8192,
micro-batch 4 per GPU) and ``mal760m`` (TitansMAL, dim 1536, 24 layers, 16
heads of 96, window 1024, L_M=3; sequence 16384, micro-batch 1 per GPU, with
activation checkpointing).  For N > 1 this framework runs its fused
data-parallel engine (replicated weights, optimizer state sharded over the
ranks); the reference arm averages gradients with one NCCL all-reduce after
backward (its own DDP setting raises, and DDP with unused-parameter search
stalls).

For N > 1 launch one process per GPU with torchrun (RANK/LOCAL_RANK/WORLD_SIZE
from the environment).  Rank 0 prints one JSON line.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize(), timed with CUDA events on the launching stream; the
max over ranks is reported.  Every step's working set (0.49 GB of weights plus
activations of several GB) is far larger than the 126 MB L2, so no extra L2
flush is inserted.  The end-to-end number ("e2e") times the public training
API (Trainer.train_step) with a pinned-host -> device copy of the step's token
ids and labels and a device -> host read of the loss in every step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tokens/sec/box (device-timed, max over ranks) at 1/2/4/8 B200 vs ref build"
MODEL_FIELDS = dict(vocab_size=32000, dim=768, num_layers=12, num_heads=12, window_size=512,
                    num_memory_layers=2, memory_hidden_mult=4.0, ffn_mult=4.0,
                    num_persistent_tokens=4, conv_kernel_size=4, use_conv=True, use_rope=True,
                    dropout=0.0, max_seq_len=4096, init_std=0.02)
SEQ, MICRO_BATCH = 4096, 8
CONFIGS = {
    "mag170m": dict(model="mag", fields=MODEL_FIELDS, seq=4096, micro_batch=8, ckpt=False,
                    desc="TitansMAG ~170M ({p:.1f}M params; dim 768, 12 layers, 12 heads, window 512, L_M=2, "
                         "4 persistent tokens, vocab 32000)"),
    "mac400m": dict(model="mac", fields=dict(vocab_size=32000, dim=1024, num_layers=24, num_heads=16,
                                             chunk_size=512, window_size=512, num_memory_layers=2,
                                             memory_hidden_mult=4.0, ffn_mult=4.0, num_persistent_tokens=16,
                                             conv_kernel_size=4, use_conv=True, use_rope=True, dropout=0.0,
                                             max_seq_len=8192, init_std=0.02),
                    seq=8192, micro_batch=4, ckpt=False,
                    desc="TitansMAC ~400M ({p:.1f}M params; dim 1024, 24 layers, 16 heads, segment 512, "
                         "16 persistent tokens, L_M=2, vocab 32000)"),
    "mal760m": dict(model="mal", fields=dict(vocab_size=32000, dim=1536, num_layers=24, num_heads=16,
                                             window_size=1024, chunk_size=1024, num_memory_layers=3,
                                             memory_hidden_mult=4.0, ffn_mult=4.0, num_persistent_tokens=4,
                                             conv_kernel_size=4, use_conv=True, use_rope=True, dropout=0.0,
                                             max_seq_len=16384, init_std=0.02),
                    seq=16384, micro_batch=1, ckpt=True,
                    desc="TitansMAL ~760M ({p:.1f}M params; dim 1536, 24 layers, 16 heads of 96, window 1024, "
                         "L_M=3, vocab 32000; activation checkpointing)"),
}
LR, BETAS, WD, CLIP = 4e-4, (0.9, 0.95), 0.1, 1.0
CFG = None


# ---------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """Samples nvidia-smi SM clocks / throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [x for x in sm if smax and x > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_batches(world, rank, steps, seed=0):
    """Synthetic uniform token ids (pinned host memory), distinct per rank and step."""
    g = torch.Generator().manual_seed(seed + 1000 * rank)
    data = torch.randint(0, MODEL_FIELDS["vocab_size"], (steps, MICRO_BATCH, SEQ + 1), generator=g)
    out = []
    for s in range(steps):
        ids = data[s, :, :-1].contiguous().pin_memory()
        lab = data[s, :, 1:].contiguous().pin_memory()
        out.append({"input_ids": ids, "labels": lab})
    return out


def count_launches(step_fn, prefixes) -> tuple[int, int]:
    """(our kernels, all kernels) launched by one call of step_fn (counted with the profiler,
    outside the timed region)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    ours = total = 0
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        name = e.name
        if "memcpy" in name.lower() or "memset" in name.lower():
            continue
        total += 1
        if any(p in name for p in prefixes):
            ours += 1
    return ours, total


# ---------------------------------------------------------------------------- arms
def build_ours(device, world, parallel="dp", overlap=True, reshard=True, wavefront=0):
    from titans_pytorch_b200 import TitansConfig, create_model
    from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig
    from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

    torch.manual_seed(0)
    model = create_model(CFG["model"], TitansConfig(**MODEL_FIELDS))
    if CFG["ckpt"]:
        enable_gradient_checkpointing(model)
    if wavefront > 1 and CFG["model"] == "mac":
        from titans_pytorch_b200.utils.perf import enable_wavefront

        enable_wavefront(model, wavefront)
    engine = None
    if world > 1 and parallel == "fsdp":
        from titans_pytorch_b200.parallel.fsdp import FullyShardedEngine

        engine = FullyShardedEngine(reshard=reshard, overlap=overlap)
    elif world > 1:
        from titans_pytorch_b200.parallel.ddp import DataParallelEngine

        engine = DataParallelEngine(overlap=overlap)
    # the whole step (with the fused data-parallel reduce/update for N > 1) is
    # captured in a CUDA graph: two eager warm-up steps, the capture on the third
    # warm-up call, replays in the timed region
    tr = Trainer(model, TrainStepConfig(lr=LR, betas=BETAS, weight_decay=WD, grad_clip=CLIP,
                                        cuda_graph=True, graph_warmup=2),
                 device=device, engine=engine)
    nparams = sum(p.numel() for p in tr.optimizer.space.params)
    return tr, nparams


def build_reference(device, world, local, mode="as-shipped"):
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "titans")):
        return None, "reference not installed under baseline/_ref"
    sys.path.insert(0, ref_dir)
    import titans  # the reference package, unmodified

    if mode == "grad-correct":
        # The shipped package calls raw Triton RMSNorm / SiLU-mul kernels without
        # a backward on CUDA (src/titans/models.py:61-63, 105-111), so only the
        # embedding trains.  Switching its Triton probe off before the first
        # forward (a runtime flag, no source edit) makes it take its own PyTorch
        # fallbacks: the same math as this framework's step, gradients included.
        import titans.triton_kernels as tk

        tk.HAS_TRITON = False

    torch.manual_seed(0)
    cls = {"mag": titans.TitansMAG, "mac": titans.TitansMAC, "mal": titans.TitansMAL}[CFG["model"]]
    model = cls(titans.TitansConfig(**MODEL_FIELDS))
    # the reference trainer's bf16 mode: the whole model in bf16 (scripts/pretrain.py:460-463)
    model = model.to(device=device, dtype=torch.bfloat16)
    nparams = sum(p.numel() for p in model.parameters())
    # No activation checkpointing on this arm: the reference's own
    # enable_gradient_checkpointing (optimized_training.py:428-457) fails in the
    # recompute (its memory update runs torch.autograd.grad inside the
    # checkpointed block, so the recomputed graph differs); without it the arm
    # only skips recomputation.
    # Data parallel for N > 1: gradients averaged with one flat NCCL all-reduce
    # after backward.  The reference's own DDP setting (find_unused_parameters=
    # False) raises at the second iteration, and DDP with find_unused_parameters=
    # True stalls in an all-reduce (its memory update calls torch.autograd.grad
    # inside the forward); FSDP would shard the parameters its memory update
    # rewrites through .data.
    params = [p for p in model.parameters() if p.requires_grad]

    def allreduce_grads():
        import torch.distributed as dist

        grads = [p.grad for p in params if p.grad is not None]
        flat = torch._utils._flatten_dense_tensors(grads)
        dist.all_reduce(flat)
        flat.div_(world)
        for g, f in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
            g.copy_(f)

    opt = torch.optim.AdamW(model.parameters(), lr=LR, betas=BETAS, weight_decay=WD, fused=True)

    class RefStep:
        def __init__(self):
            self.model, self.opt = model, opt

        def train_step(self, batch):
            ids = batch["input_ids"].to(device, non_blocking=True)
            lab = batch["labels"].to(device, non_blocking=True)
            logits, _ = self.model(ids)
            loss = torch.nn.functional.cross_entropy(logits.view(-1, logits.size(-1)), lab.view(-1))
            loss.backward()
            if world > 1:
                allreduce_grads()
            torch.nn.utils.clip_grad_norm_(model.parameters(), CLIP)
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
            return loss.detach()

    return (RefStep(), nparams), None


# ---------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-mode", choices=["as-shipped", "grad-correct"], default="as-shipped",
                    help="reference arm: the package as shipped (its Triton RMSNorm / SiLU-mul cut the gradient, "
                         "so only the embedding trains), or with its Triton probe off (full gradients)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="mag170m")
    ap.add_argument("--parallel", choices=["dp", "fsdp"], default="dp",
                    help="N > 1, this framework: dp = replicated weights, optimizer state sharded; fsdp = "
                         "parameters sharded per block, all-gathered inside the first GEMM of the previous block")
    ap.add_argument("--overlap", choices=["auto", "on", "off"], default="auto",
                    help="N > 1, this framework: reduce-scatter each block's gradients on a communication stream "
                         "during the backward (on) or after it (off); auto = off for dp (measured faster), on "
                         "for fsdp")
    ap.add_argument("--fsdp-mode", choices=["full", "grad-op"], default="full",
                    help="fsdp: full = FULL_SHARD (parameters gathered per use into working slots, gradients "
                         "reduce-scattered per block during the backward); grad-op = SHARD_GRAD_OP (gathered "
                         "parameters kept until the step)")
    ap.add_argument("--wavefront", type=int, default=-1,
                    help="mac400m: run the (layer, segment) loop as a wavefront on this many CUDA streams "
                         "(0 = sequential; default: 2 on one GPU, 0 with several; dp without overlap also "
                         "takes it, fsdp does not)")
    args = ap.parse_args()
    global CFG, MODEL_FIELDS, SEQ, MICRO_BATCH
    CFG = CONFIGS[args.config]
    MODEL_FIELDS, SEQ, MICRO_BATCH = CFG["fields"], CFG["seq"], CFG["micro_batch"]
    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun for N>1")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    init_dist(world, local)
    device = torch.device("cuda", local)
    K, W = args.steps, max(3, args.warmup)

    if args.impl == "reference":
        built, why = build_reference(device, world, local, args.ref_mode)
        if built is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            return
        trainer, nparams = built
        prefixes = ()
    else:
        overlap = args.overlap == "on" or (args.overlap == "auto" and args.parallel == "fsdp")
        if args.wavefront < 0:
            args.wavefront = 2 if world == 1 else 0  # measured on one GPU; ask for it explicitly with dp
        trainer, nparams = build_ours(device, world, args.parallel, overlap=overlap,
                                      reshard=args.fsdp_mode == "full", wavefront=args.wavefront)
        prefixes = ("tb::",)

    batches = make_batches(world, rank, W + K + 1)
    dev_batches = [{k: v.to(device) for k, v in b.items()} for b in batches]

    # warm-up
    for i in range(W):
        trainer.train_step(dev_batches[i])
    torch.cuda.synchronize()

    # device-timed region: K steps on device-resident inputs
    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                           if "CUDA_VISIBLE_DEVICES" in os.environ else local)
    barrier(world)
    torch.cuda.synchronize()
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(K):
        loss = trainer.train_step(dev_batches[W + i])
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / K
    ms = max_over_ranks(ms, world)
    final_loss = float(loss)

    # end-to-end through the public API: pinned H2D inputs + D2H loss every step
    e2e = None
    if not args.no_e2e:
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for i in range(K):
            l = trainer.train_step(batches[W + i])
            float(l)  # device -> host read of the step's loss
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1000 / K
        ems = max_over_ranks(e0.elapsed_time(e1) / K, world)
        tok = world * MICRO_BATCH * SEQ
        bi = batches[0]["input_ids"].numel() * batches[0]["input_ids"].element_size() * 2
        e2e = {"value": tok / (ems / 1000), "unit": "tokens/s", "ms_per_step": ems, "wall_ms_per_step": wall,
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4}

    # launch count of one extra (untimed) step; every rank takes it, so the ranks'
    # collectives stay matched
    ours, total = count_launches(lambda: trainer.train_step(dev_batches[-1]), prefixes)

    tokens = world * MICRO_BATCH * SEQ
    value = tokens / (ms / 1000)
    parallelism = f"dp{world}"
    overlapped = args.overlap == "on" or (args.overlap == "auto" and args.parallel == "fsdp")
    when = "per block during the backward" if overlapped else "after the backward"
    if world > 1:
        parallelism = (f"dp{world} (grads all-reduced after backward)" if args.impl == "reference"
                       else (f"fsdp{world} ({'FULL_SHARD: parameters gathered per use into working slots' if args.fsdp_mode == 'full' else 'SHARD_GRAD_OP'}; "
                             f"all-gather fused into the previous block's first tcgen05 GEMM; peer-memory "
                             f"reduce-scatter {when}; fused AdamW shard)")
                       if args.parallel == "fsdp"
                       else f"dp{world} (peer-memory reduce-scatter {when}; fused AdamW shard / all-gather)")
    if args.impl == "ours" and args.wavefront > 1 and CFG["model"] == "mac":
        parallelism += f"; (layer, segment) wavefront on {args.wavefront} streams"
    peak = torch.cuda.max_memory_allocated(device)
    comm = getattr(getattr(trainer, "optimizer", None), "comm_bytes", None)
    peak_gib = (peak + (comm() if comm is not None else 0)) / 2 ** 30
    peak_gib = max_over_ranks(peak_gib, world)
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic uniform token ids, random init (std 0.02)",
            "config": {"model": CFG["desc"].format(p=nparams / 1e6),
                       "global_batch": MICRO_BATCH * world, "seq_len": SEQ, "parallelism": parallelism,
                       "l2": "no flush: per-step working set (weights + activations, several GB) >> 126 MB L2"},
            "clocks": clocks, "e2e": e2e, "gpu_launches": ours * K, "all_launches_per_step": total,
            "final_loss": final_loss,
            "peak_mem_gib": round(peak_gib, 2),
        }
        if args.impl == "reference":
            out["impl"] = "reference"
            out["reference_mode"] = (("as shipped" if args.ref_mode == "as-shipped" else
                                      "gradient-correct (titans.triton_kernels.HAS_TRITON = False at run time: "
                                      "PyTorch RMSNorm / SiLU-mul with gradients)")
                                     + ": unmodified package, bf16 model (scripts/pretrain.py:460), "
                                     "fused AdamW, clip 1.0; for N>1 grads averaged by one flat NCCL all-reduce "
                                     "after backward (its DDP raises or stalls)"
                                     + ("; activation checkpointing off (the reference's own "
                                        "enable_gradient_checkpointing fails in its recompute)" if CFG["ckpt"] else ""))
        else:
            out["impl"] = "ours"
        print(json.dumps(out))
    if world > 1:
        import torch.distributed as dist

        if hasattr(trainer, "_graph"):
            trainer._graph = None  # release the captured step before the group goes away
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
