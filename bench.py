"""Benchmark: midpoint-reversible training of the 20.3M decoder (BASELINE cfg2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--method midpoint|euler]
    torchrun --nproc-per-node N bench.py --gpus N ...      (data parallel, NCCL)
    python bench.py --impl reference ...                   (the reference's CPU path)

A step is one optimizer update of cfg2 per GPU: physical batch 29x512,
gradient accumulation 2 (29,696 targets per GPU), bf16 autocast semantics with
fp32 parameters and residual stream, AdamW(0.9, 0.95, wd 0.1), clip 1.0, on the
seeded Zipf/EOS synthetic token stream (the FineWeb-Edu file is not available;
the stream has its vocabulary, EOS convention and uint16 format). Weak scaling:
every rank processes its own 29,696 targets per update.

Prints ONE JSON line (rank 0). `value` is the device-timed, whole-job
throughput with the update's token batches already in HBM (staged into the
update's input buffers by device copies inside the timed region); `e2e` is the
same metric through the public trainer API with the batches copied from pinned
host memory and the loss read back to the host every step.
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
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train targets/sec (midpoint, 20.3M model)"


def metric_name(method: str, model: str = "cfg2") -> str:
    """BASELINE's metric; the Euler configuration (cfg3) names its recurrence
    and the scaled configuration (cfg5) its model."""
    name = METRIC if method == "midpoint" else METRIC.replace("midpoint", method)
    return name if model == "cfg2" else name.replace("20.3M", MODELS[model]["name"])
UNIT = "targets/s"
FLOP_PER_TARGET = 143_255_040  # 4 x body (fwd + attention) + 3 x head, cfg2 (20.3M model)

# The benchmarked model shapes: cfg2/cfg3 (the 20.3M decoder, BASELINE configs[1]/[2])
# and cfg5 (the scaled decoder). FLOP per target is the
# midpoint-reversible minimum: 4 x (body GEMMs + causal attention) + 3 x head.
MODELS = {
    "cfg2": dict(config={}, batch=29, seq=512, accumulation=2, flop=FLOP_PER_TARGET, name="20.3M",
                 shape="L7 d256 H8 ff1024 V50257 T512"),
    "cfg5": dict(config=dict(n_layers=24, d_model=1024, n_heads=16, d_ff=4096, max_sequence_length=2048),
                 batch=16, seq=2048, accumulation=1, flop=3_932_657_664, name="456M scaled",
                 shape="L24 d1024 H16 ff4096 V50257 T2048"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["librevk", "reference"], default="librevk")
    ap.add_argument("--method", choices=["midpoint", "euler"], default="midpoint")
    ap.add_argument("--model", choices=sorted(MODELS), default="cfg2",
                    help="cfg2: the 20.3M decoder (default); cfg5: the scaled 24-layer d1024 decoder")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--accumulation", type=int, default=None)
    ap.add_argument("--no-graph", action="store_true", help="run updates eagerly instead of replaying a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--forward-overlap", choices=["start", "head", "after_head"], default="start",
                    help="start the later microsteps' forward sweeps beside microstep 0's (default), or "
                         "microstep m+1's beside microstep m's head GEMM, or after it")
    ap.add_argument("--no-tied-split", action="store_true",
                    help="data parallel: reduce the tied embedding gradient as one bucket after the sweep")
    ap.add_argument("--reference-memory", action="store_true",
                    help="measure the reference's own peak allocated HBM at this shape (needs baseline/_ref)")
    args = ap.parse_args()
    spec = MODELS[args.model]
    for key in ("batch", "seq", "accumulation"):
        if getattr(args, key) is None:
            setattr(args, key, spec[key])
    return args


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def config_block(args, world):
    spec = MODELS[args.model]
    tag = args.model if not (args.model == "cfg2" and args.method == "euler") else "cfg3"
    return {"workload": f"{tag}: {args.method}-reversible {spec['name']} decoder ({spec['shape']}), "
                        f"batch {args.batch}x{args.seq} x accumulation {args.accumulation} per GPU, bf16 autocast, "
                        f"AdamW(0.9,0.95,wd0.1) clip 1.0",
            "method": args.method, "global_batch": args.batch * args.accumulation * world,
            "seq_len": args.seq, "parallelism": f"dp{world}",
            "targets_per_update_per_gpu": args.batch * args.seq * args.accumulation,
            "l2": f"inputs larger than L2 (per-step working set: "
                  f"{args.batch * args.seq * 50304 * 2 / 1e9:.1f} GB logits + the parameter state)"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.first = threading.Event()
        self.start = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            # nvidia-smi can take longer to start than the timed region lasts:
            # the region begins once it is sampling
            self.first.wait(timeout=10.0)
            self.start = len(self.lines)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.first.set()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # samples taken during the region; the last one before it if the region
        # was shorter than the sampling interval
        lines = self.lines[self.start:] or self.lines[max(self.start - 1, 0):self.start]
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ CPU baseline (oracle port)
def _cpu_trainer(method: str, batch: int, seq: int, accumulation: int, updates: int):
    """The reference's pure-PyTorch fp32 CPU update (forward + reconstruction
    backward + clip + AdamW, restated in oracle/), on every host thread, over
    the benchmark's own update shape, one microstep at a time: returns
    (threads, microstep) where microstep() runs the next batch x seq microstep
    of the seeded stream (the clip + AdamW step after every `accumulation`-th)
    and returns its target count."""
    from oracle import model as om, stream as ost
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = om.Config()
    tr = om.Trainer(om.init_params(cfg, seed=1337), cfg, om.TrainConfig(), method, eps=1e-6)
    per_update = batch * seq * accumulation
    data = ost.synthetic_stream(per_update * (updates + 1) + 1, seed=1337)
    state = {"committed": 0, "m": 0, "loss": 0.0}

    def microstep():
        c0, m = state["committed"], state["m"]
        if m == 0:
            tr.opt.zero_grad(set_to_none=True)
            state["loss"] = 0.0
        x, y, n = ost.batch_at(data, c0 + m * batch * seq, batch, seq, c0 + per_update)
        state["loss"] += tr.microstep(x, y, per_update)
        if m + 1 == accumulation:
            tr.finish(c0, per_update, state["loss"])
            state["committed"], state["m"] = c0 + per_update, 0
        else:
            state["m"] = m + 1
        return n

    return threads, microstep


def cpu_baseline(method: str, batch: int, seq: int, accumulation: int):
    """The reference's CPU path timed on this host's cores on a bounded sample
    of the benchmark's own workload (about 10-30 s): after one warm-up
    microstep, the timed sample is the rest of that update — the next
    batch x seq microsteps through the clip + AdamW step."""
    threads, microstep = _cpu_trainer(method, batch, seq, accumulation, 1)
    microstep()  # warm-up
    n = max(accumulation - 1, 1)
    start = time.perf_counter()
    targets = sum(microstep() for _ in range(n))
    el = time.perf_counter() - start
    return {"value": targets / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} microstep(s) of {batch}x{seq} targets closing an update of accumulation {accumulation} "
                      f"(clip + AdamW included; the benchmarked update shape) after a warm-up microstep, fp32, full "
                      f"20.3M model, oracle port of ReversibleLM + _InverseStack + AdamW on {threads} host threads, "
                      f"{el:.1f} s"}


def reference_arm(args):
    """The reference's CPU implementation of the path (the oracle port), rank 0
    only. Each step is one microstep of the benchmark's update (batch x seq
    targets; the clip + AdamW step closes every accumulation-th), so K steps
    time K / accumulation updates of the benchmarked shape within minutes."""
    rank, world, _ = env_rank()
    if rank != 0:
        return
    if args.model != "cfg2":
        print(json.dumps({"impl": "reference", "unavailable": f"the CPU port of the reference path is timed on the "
                          f"20.3M model only; one {args.model} microstep takes minutes on the host cores"}))
        return
    total = args.steps + args.warmup
    threads, microstep = _cpu_trainer(args.method, args.batch, args.seq, args.accumulation,
                                      total // args.accumulation + 1)
    for _ in range(args.warmup):
        microstep()
    t0 = time.perf_counter()
    targets = sum(microstep() for _ in range(args.steps))
    el = time.perf_counter() - t0
    value = targets / el
    line = {"metric": metric_name(args.method), "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el / max(args.steps, 1) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_block(args, world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"each step: one {args.batch}x{args.seq} microstep of the benchmarked update "
                                       f"(accumulation {args.accumulation}; clip + AdamW after every "
                                       f"{args.accumulation}th), fp32 CPU oracle port of the reference path, "
                                       f"{threads} threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_memory(args):
    """Peak allocated HBM of the REFERENCE's own training microsteps on cuda:0
    at the benchmark's shape (train_baseline.py:256-280 under bf16 autocast,
    accumulation included, AdamW step), for its plain reversible trainer path
    (ReversibleLM + full-logit F.cross_entropy) and its optimised path
    (install_v3(core_mode='split', mlp_tokens=8192) + cached_head_backward with
    1024-token chunks; Triton options off). Needs the unmodified reference
    package installed under baseline/_ref; prints one JSON line."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "reversibility").is_dir():
        print(json.dumps({"reference_peak_alloc": "unavailable", "why": "baseline/_ref holds no reference install"}))
        return
    sys.path.insert(0, str(ref_dir))
    import torch.nn.functional as F
    from reversibility import ModelConfig, ReversibleLM
    from reversibility.optimized_v3 import cached_head_backward, install_v3
    from reversability_b200 import data as rdata
    dev = torch.device("cuda", 0)
    B, T, acc = args.batch, args.seq, args.accumulation
    stream = rdata.synthetic_stream(B * T * acc + 1, seed=1337)
    batches, targets = rdata.update_batches(stream, 0, 0, 1, B, T, acc, len(stream) - 1)
    out = {}
    for path in ("reversible_trainer", "optimized_split_tiled_cached_head"):
        torch.manual_seed(1337)
        model = ReversibleLM(ModelConfig(**MODELS[args.model]["config"]), args.method).to(dev)
        if path != "reversible_trainer":
            install_v3(model, core_mode="split", mlp_tokens=8192)
        opt = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(dev)
        for x, y, _ in batches:
            x, y = x.to(dev), y.to(dev)
            if path == "reversible_trainer":
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    logits = model(x)
                    loss = F.cross_entropy(logits.flatten(0, 1), y.flatten(), ignore_index=-100, reduction="sum")
                    (loss / targets).backward()
                del logits, loss
            else:
                cached_head_backward(model, x, y, targets, 1024, precision="bf16")
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        torch.cuda.synchronize()
        out[path] = torch.cuda.max_memory_allocated(dev)
        del model, opt
        torch.cuda.empty_cache()
    print(json.dumps({"reference_peak_alloc_bytes": out, "config": config_block(args, 1),
                      "device": torch.cuda.get_device_name(dev)}), flush=True)


# ------------------------------------------------------------------ dominant-kernel roofline
PROFILES = Path(__file__).resolve().parent / "profiles"


def profiled_traffic(name: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of
    one ncu capture) recorded in profiles/ as `traffic_bytes_per_launch[name]: N`."""
    for f in sorted(PROFILES.glob("*.md")):
        for line in f.read_text().splitlines():
            if line.startswith(f"traffic_bytes_per_launch[{name}]:"):
                return int(line.split(":", 1)[1].strip())
    return None


def kernel_roofline(trainer, peak_tflops):
    """The dominant kernel of the step, the head GEMM with the log-sum-exp
    epilogue ([29*512, 256] x [256, 50257] bf16, rk_head_fprop), timed live:
    CUDA event record nodes around it inside the captured update, read after
    the timed region (both microsteps of the last update). Falls back to
    timing it alone when the trainer runs the fp32 path."""
    M, V, d = trainer.M, trainer.cfg.vocab_size, trainer.cfg.d_model
    flops = 2.0 * M * V * d
    durations = trainer.head_fprop_ms()
    if durations:
        ms = sum(durations) / len(durations)
        how = "event nodes around it in the timed CUDA graph (last update, %d launches)" % len(durations)
    else:
        from reversability_b200 import functional as fn
        hidden = torch.randn(M, d, device=trainer.dev).to(trainer.cd)
        out = trainer.logits[:, :V]
        s = torch.cuda.current_stream()
        for _ in range(5):
            fn.linear_fwd(hidden, trainer.tok_c, out=out)
        n = 20
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(s)
        for _ in range(n):
            fn.linear_fwd(hidden, trainer.tok_c, out=out)
        stop.record(s)
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop) / n
        how = "alone, 20 launches"
    achieved = flops / (ms * 1e-3) / 1e12
    return {"kernel": "gemm_tc_kernel EPI_LSE (rk_head_fprop, M=%d N=%d K=%d, bf16)" % (M, V, d),
            "bound": "tensor", "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
            "frac": achieved / peak_tflops, "avg_launch_us": ms * 1e3, "flops_per_launch": flops,
            "timed": how,
            # the committed capture is of the cfg2 shape (M 14,848, K 256); other shapes have none
            "traffic": profiled_traffic("rk_head_fprop") if (M, d) == (14848, 256) else None}


# ------------------------------------------------------------------ main arm
def main():
    args = parse()
    if args.reference_memory:
        reference_memory(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    rank, world, local = env_rank()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("run N>1 under torchrun (one process per GPU)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist.group.WORLD

    import reversability_b200 as rb
    from reversability_b200 import _lib, data as rdata
    from reversability_b200.train import ReversibleTrainer, TrainSettings, learning_rate

    s = TrainSettings(batch_size=args.batch, sequence_length=args.seq, accumulation=args.accumulation,
                      tied_split=not args.no_tied_split, forward_overlap=args.forward_overlap)
    torch.manual_seed(1337)
    spec = MODELS[args.model]
    model = rb.ReversibleLM(rb.ModelConfig(**spec["config"]), args.method).to(dev)
    trainer = ReversibleTrainer(model, s, pg)
    per_update = args.batch * args.seq * args.accumulation
    total_updates = args.warmup + 2 * args.steps + 2
    stream = rdata.synthetic_stream(per_update * world * total_updates + 1, seed=1337)
    limit = len(stream) - 1

    def host_batches(u):
        committed = u * per_update * world
        b, targets = rdata.update_batches(stream, committed, rank, world, args.batch, args.seq, args.accumulation,
                                          limit)
        return committed, b, targets

    # device copies of the device loop's batches (the e2e loop reads the
    # memory-mapped stream file through the trainer's pinned prefetcher)
    first_e2e_update = args.warmup + 1 + args.steps
    pinned, resident = [], []
    for u in range(first_e2e_update):
        committed, b, targets = host_batches(u)
        ids = torch.stack([x for x, _, _ in b])
        lab = torch.stack([y for _, y, _ in b])
        pinned.append((committed, ids, lab, targets))
        resident.append((ids.to(dev), lab.to(dev)))
    torch.cuda.synchronize()

    def stage_device(u):
        _, _, _, targets = pinned[u]
        trainer.ids.copy_(resident[u][0])
        trainer.labels.copy_(resident[u][1])
        trainer.inv_denominator.fill_(1.0 / targets)

    def lr_of(u):
        committed, _, _, targets = pinned[u]
        return learning_rate(s, committed, targets)

    # warm-up (eager), then capture one update as a CUDA graph
    stage_device(0)
    launches_before = _lib.launch_count()
    trainer.update(lr_of(0))
    launches_per_update = _lib.launch_count() - launches_before
    if trainer.fused_head:
        trainer.time_head_fprop()
    use_graph = not args.no_graph
    if use_graph:
        try:
            trainer.capture(warmup=1)
        except Exception as exc:  # capture unsupported in this process setup: run the same updates eagerly
            trainer.graph = None
            use_graph = False
            if rank == 0:
                print(f"# CUDA graph capture failed ({exc!r}); timing eager updates", file=sys.stderr)
    for u in range(1, args.warmup + 1):
        stage_device(u)
        trainer.update(lr_of(u))
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # ---- device-resident timed region
    first = args.warmup + 1
    cs = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:  # sampling before the barrier, so every rank starts together
        barrier()
        torch.cuda.synchronize()
        clocks.start = len(clocks.lines)
        start.record(cs)
        for k in range(args.steps):
            u = first + k
            stage_device(u)
            trainer.update(lr_of(u))
        stop.record(cs)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(stop)
    ms_max = ms
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = t.item()
    value = per_update * world * args.steps / (ms_max / 1e3)
    peak_alloc = torch.cuda.max_memory_allocated(dev)

    # ---- end-to-end timed region through the trainer API: the token stream as
    # a uint16 file, memory-mapped; each update's batches built by the
    # prefetch thread into pinned buffers, copied host -> device inside
    # train(); the loss sum copied back to the host every step
    import tempfile
    losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    tmpdir = tempfile.TemporaryDirectory(prefix="revk_stream_")
    mm = rdata.open_stream(rdata.write_stream(Path(tmpdir.name) / "train.bin", stream))
    e2e_start = first_e2e_update * per_update * world
    prefetch = rdata.UpdatePrefetcher(mm, rank, world, args.batch, args.seq, args.accumulation,
                                      min(limit, e2e_start + args.steps * per_update * world), start=e2e_start)
    h2d = 2 * args.accumulation * args.batch * args.seq * 8  # ids + labels, int64

    def keep_loss(k, staged, loss):
        losses[k].copy_(loss, non_blocking=True)

    barrier()
    torch.cuda.synchronize()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(cs)
    ran = trainer.train(prefetch, max_updates=args.steps, on_update=keep_loss)
    e_stop.record(cs)
    torch.cuda.synchronize()
    barrier()
    prefetch.close()
    tmpdir.cleanup()
    if ran != args.steps:
        raise RuntimeError(f"the e2e loop ran {ran} of {args.steps} updates")
    e_ms = e_start.elapsed_time(e_stop)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = t.item()
    e2e_value = per_update * world * args.steps / (e_ms / 1e3)
    status = _lib.device_status()
    finite = bool(torch.isfinite(losses).all())

    if rank == 0:
        hbm, tflops, tflops_sus, peak_kind = measured_peaks()
        roof = kernel_roofline(trainer, tflops)
        roof["peak_source"] = peak_kind
        model_flops = value * spec["flop"] / world / 1e12
        line = {
            "metric": metric_name(args.method, args.model), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_block(args, world),
            "roofline": roof,
            "model_roofline": {"achieved": model_flops, "peak": tflops_sus or tflops, "unit": "TFLOP/s per GPU",
                               "frac": model_flops / (tflops_sus or tflops),
                               "flop_per_target": spec["flop"], "peak_source": peak_kind + " sustained"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                    "path": "ReversibleTrainer.train over data.UpdatePrefetcher (memory-mapped uint16 stream, "
                            "pinned buffers filled by a background thread)"},
            "gpu_launches": launches_per_update * args.steps,
            "launches_per_update": launches_per_update,
            "cuda_graph": use_graph,
            "peak_alloc_bytes": peak_alloc,
            "clocks": clocks.summary(),
            "loss_first_last": [float(losses[0]) / per_update / world, float(losses[-1]) / per_update / world],
            "losses_finite": finite, "device_status": status,
        }
        if not args.no_cpu_baseline and world == 1 and args.model == "cfg2":
            line["cpu_baseline"] = cpu_baseline(args.method, args.batch, args.seq, args.accumulation)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        trainer.graph = None
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
