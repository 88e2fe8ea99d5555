#!/usr/bin/env python3
"""Benchmark of the B200 forward pass (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C5] [--impl b200|reference]
                    [--scaling strong|weak]

Workload: BASELINE configuration C5 by default (batch 512, seq 1024,
d_model 256, 8 heads, ffn 1024, 4 layers, causal), the configuration the
metric's 1/2/4/8-GPU clause is quoted on.  One process per GPU (torchrun for
N > 1).  Strong scaling (default): the one batch of 512 sequences is split
into contiguous slices (sharding.shard_bounds, 64 per GPU at N = 8), every
rank runs its slice, and every slice's FP32 output is pushed into one gather
buffer on GPU 0 (tt_model_forward_gather: NVLink copies on the copy engines,
each overlapped with the next step's compute).  A step is one forward of this
rank's slice plus its push.

  value  device-resident inputs; per step: L2 flush (256 MiB write, untimed),
         CUDA events around the forward and its push; after the last step the
         wait for the last push is timed too; max over ranks of the summed
         times; sequences/s of the whole batch.  compute_only (no push),
         latency_ms (one step with its push waited for) and weak (every rank a
         whole batch of its own, nothing gathered) are reported beside it, and
         gather_check says whether rank 0's gathered batch equals, bit for bit,
         its own 1-GPU forward of the whole batch.
  e2e    same metric through the public model call with host buffers
         (model.forward_host -> tt_model_forward_host): every step copies the
         input slice from pinned host memory and the FP32 output back to host
         memory inside the timed region, the copies overlapped with the
         kernels by batch chunks; with N > 1 every rank writes its slice into
         one page-locked host buffer shared with rank 0's process.
  roofline  the dominant kernel's algorithmic FLOPs (or bytes) per launch over
         its mean event-timed duration (events the library records around every
         launch, on the launch stream) in a profiled pass of the same K steps
         run right after the timed ones, against the measured peak in
         MEASURED_PEAKS.json.  The timed steps themselves run without those
         events, which would keep consecutive kernels from overlapping their
         set-up (programmatic dependent launch).
  cpu_baseline  (rank 0, N = 1) the FP32 oracle on the host cores, on a
         bounded sample of sequences of the same workload.

--impl reference times the reference's FP32 CPU path (the oracle
restatement; the reference itself is Python that cannot be installed on the
GPU box) on rank 0 only, a bounded sample of sequences per step.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Workload table: (batch, seq, d_model, heads, ffn, layers, causal, padding_ratio)
WORKLOADS = {
    "C1": (64, 128, 128, 4, 128, 4, True, 0.0),
    "C2": (64, 1024, 128, 4, 128, 4, True, 0.0),
    "C3": (256, 256, 32, 2, 128, 4, True, 0.0),
    "C4": (16, 2048, 512, 8, 2048, 6, True, 0.5),
    "C5": (512, 1024, 256, 8, 1024, 4, True, 0.0),
    # The reference suite's other cases (analysis_profile_mixed.py:20-26), every token valid.
    "S6": (10000, 128, 128, 4, 128, 4, True, 0.0),
    "S8": (64, 128, 1024, 4, 1024, 4, True, 0.0),
    "S10": (64, 128, 128, 2, 128, 4, True, 0.0),
    "S11": (64, 128, 128, 16, 128, 4, True, 0.0),
    "S13": (64, 1024, 128, 4, 128, 4, True, 0.0),
}
METRIC = "sequences/sec (forward, FP32 in/out)"
UNIT = "seq/s"
SEED = 1234 + 100000  # the reference's timing-input seed (torch_transformer_benchmark.py:747)
KERNEL_KIND_LABEL = {"qkv": "gemm_kernel<EPI_QKV>", "out_ln": "gemm_kernel<EPI_RESID_LN>",
                     "ffn_in": "gemm_kernel<EPI_GELU>", "ffn_out_ln": "gemm_kernel<EPI_RESID_LN>",
                     "ln0": "layernorm_rows_kernel", "mask": "mask_kv_end_kernel"}


def kernel_label(kind, cfg):
    """Name of the kernel a kind of launch runs for this shape (the library's dispatch)."""
    hd = cfg["d_model"] // cfg["heads"]
    if kind == "attn":
        if hd == 8:
            return "attn_db_fwd_kernel<16> (head_dim 8 stored 16 wide)"
        return f"attn_db_fwd_kernel<{hd}>"
    if kind == "ffn_fused":
        return f"ffn2_kernel<{cfg['d_model']}>" if cfg["d_model"] in (128, 256) else f"ffn_fused_kernel<{cfg['d_model']}>"
    return KERNEL_KIND_LABEL.get(kind, kind)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="C5", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-seconds", type=float, default=12.0)
    ap.add_argument("--chunk", type=int, default=None,
                    help="sequences per chunk of the host-buffer pipeline (e2e); default: up to 8 chunks")
    ap.add_argument("--graph", action="store_true",
                    help="time replays of one captured CUDA graph of the forward (small workloads)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (smaller profiling cases)")
    ap.add_argument("--scaling", default="strong", choices=("strong", "weak"),
                    help="strong: the workload's batch split across the GPUs and gathered to GPU 0 (default); "
                         "weak: every GPU runs a whole batch of its own")
    return ap.parse_args()


def make_inputs(cfg, padding_ratio, seed):
    """x ~ N(0,1) FP32 [B, S, D] and the prefix key-padding mask, generated on CPU
    the way the reference's generate_random_case does (torch_transformer_benchmark.py:448-486)."""
    B, S, D = cfg["batch"], cfg["seq"], cfg["d_model"]
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn(B, S, D, generator=g, dtype=torch.float32)
    if padding_ratio <= 0:
        return x, None
    min_valid = max(1, int(round(S * (1.0 - padding_ratio))))
    lengths = torch.randint(min_valid, S + 1, (B,), generator=g)
    mask = torch.arange(S)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


def algorithmic(cfg, batch):
    """Per-layer algorithmic FLOPs and HBM bytes of each kernel kind for `batch` sequences.

    attention: FLOPs 2*B*S^2*D causal (4*B*S^2*D full), bytes 8ND (Q, K, V read, ctx written, FP16)
    qkv:       FLOPs 6ND^2, bytes 8ND + 6D^2
    out_ln:    FLOPs 2ND^2, bytes 12ND + 2D^2 (ctx FP16 in, residual FP32 in/out, normalized FP16 out)
    ffn (split): ffn_in FLOPs 2NDF, bytes 2ND + 2NF + 2DF; ffn_out_ln FLOPs 2NDF, bytes 2NF + 10ND + 2DF
    ffn_fused: FLOPs 4NDF, bytes 12ND + 4DF (normalized FP16 in, residual FP32 in/out, normalized out)
    """
    S, D, F = cfg["seq"], cfg["d_model"], cfg["ffn"]
    N = batch * S
    attn_flops = (2.0 if cfg["causal"] else 4.0) * batch * S * S * D
    return {
        "attn": (attn_flops, 8.0 * N * D),
        "qkv": (6.0 * N * D * D, 8.0 * N * D + 6.0 * D * D),
        "out_ln": (2.0 * N * D * D, 12.0 * N * D + 2.0 * D * D),
        "ffn_in": (2.0 * N * D * F, 2.0 * N * D + 2.0 * N * F + 2.0 * D * F),
        "ffn_out_ln": (2.0 * N * D * F, 2.0 * N * F + 10.0 * N * D + 2.0 * D * F),
        "ffn_fused": (4.0 * N * D * F, 12.0 * N * D + 4.0 * D * F),
        "ln0": (0.0, 6.0 * N * D),
        "mask": (0.0, float(batch * S)),
    }


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def load_traffic(workload, per_gpu_batch, kind):
    """DRAM bytes per launch of (workload, kernel kind) from the committed ncu summary, or None.

    The summary records bytes for a capture at `captured_batch` sequences per
    launch; traffic grows in proportion to the sequences a launch processes.
    """
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            ent = json.load(f).get(f"{workload}/{kind}")
        if ent is None:
            return None
        return float(ent["bytes_per_launch"]) * per_gpu_batch / float(ent["captured_batch"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.out = open(self.path, "w")
        self.proc = subprocess.Popen([exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)

    def stop(self, gpu_indices):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in gpu_indices:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        loaded = [v for v in sm if v > 0.5 * (mx or max(sm))] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(cfg, padding_ratio, budget_s):
    """FP32 oracle on the host cores over a bounded sample of sequences: (seq/s, cores, sample)."""
    import oracle  # the CPU baseline leg is the one place bench.py uses the oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ocfg = oracle.Config(1, cfg["seq"], cfg["d_model"], cfg["heads"], cfg["ffn"], cfg["layers"], cfg["causal"])
    sd = oracle.seeded_state_dict(ocfg, 1234)
    big = oracle.Config(cfg["batch"], cfg["seq"], cfg["d_model"], cfg["heads"], cfg["ffn"], cfg["layers"],
                        cfg["causal"])
    x, mask = make_inputs(cfg, padding_ratio, SEED)
    with torch.inference_mode():
        t0 = time.perf_counter()
        oracle.forward(sd, big, x[:1], None if mask is None else mask[:1])  # warm-up + size probe
        one = time.perf_counter() - t0
        n = int(max(1, min(cfg["batch"], budget_s / max(one, 1e-3))))
        t0 = time.perf_counter()
        done = 0
        while done < n:
            k = min(4, n - done)
            oracle.forward(sd, big, x[done:done + k], None if mask is None else mask[done:done + k])
            done += k
        dt = time.perf_counter() - t0
    return done / dt, threads, f"{done} of {cfg['batch']} sequences of the workload, batches of <=4, FP32 oracle"


def run_reference(args, cfg, padding_ratio, workload_name):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    big = oracle.Config(cfg["batch"], cfg["seq"], cfg["d_model"], cfg["heads"], cfg["ffn"], cfg["layers"],
                        cfg["causal"])
    sd = oracle.seeded_state_dict(big, 1234)
    x, mask = make_inputs(cfg, padding_ratio, SEED)
    per_step = min(4, cfg["batch"])
    times = []
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            s = (i * per_step) % max(1, cfg["batch"] - per_step + 1)
            t0 = time.perf_counter()
            oracle.forward(sd, big, x[s:s + per_step], None if mask is None else mask[s:s + per_step])
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
    total = sum(times)
    value = per_step * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name, "sample_per_step": per_step, **cfg},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} sequences per step of the {workload_name} workload, FP32 oracle "
                                   "restatement of BaselineTransformer on CPU"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class SharedHostOutput:
    """The whole batch's FP32 output in host memory shared by every rank's process.

    Rank 0 creates a file under /dev/shm; every rank maps it and page-locks its
    own slice (cudaHostRegister), so each GPU copies its slice of the output
    over its own PCIe link straight into memory rank 0 reads: the gather to
    rank 0's host needs no further copy.  Falls back to a private pinned
    buffer per rank when no shared file can be made (then ``shared`` is False).
    """

    def __init__(self, shape, s0, s1, rank, world, barrier):
        import tempfile

        self.shared = False
        self.path = None
        self._registered = None
        numel = 1
        for d in shape:
            numel *= d
        row = numel // shape[0]
        path = [None]
        if rank == 0:
            try:
                fd, p = tempfile.mkstemp(prefix="tt_b200_out_", dir="/dev/shm")
                os.close(fd)
                os.truncate(p, numel * 4)
                path[0] = p
            except OSError:
                path[0] = None
        if world > 1:
            import torch.distributed as dist

            dist.broadcast_object_list(path, src=0)
        barrier()
        self.path = path[0]
        if self.path is not None:
            try:
                full = torch.from_file(self.path, shared=True, size=numel, dtype=torch.float32).view(*shape)
                part = full[s0:s1]
                rc = torch.cuda.cudart().cudaHostRegister(part.data_ptr(), part.numel() * 4, 0)
                if int(rc) == 0:
                    self.full, self.part, self.shared = full, part, True
                    self._registered = part.data_ptr()
            except Exception:
                self.shared = False
        if not self.shared:
            self.full = None
            self.part = torch.empty((s1 - s0,) + tuple(shape[1:]), dtype=torch.float32).pin_memory()
        ok = torch.tensor([1.0 if self.shared else 0.0])
        if world > 1:
            import torch.distributed as dist

            t = ok.cuda()
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            ok = t.cpu()
        self.all_shared = bool(ok.item() > 0.5)

    def close(self, rank, barrier):
        if self._registered is not None:
            torch.cuda.cudart().cudaHostUnregister(self._registered)
            self._registered = None
        barrier()
        if rank == 0 and self.path is not None:
            try:
                os.unlink(self.path)
            except OSError:
                pass


def main() -> int:
    args = parse_args()
    B, S, D, H, F, L, causal, pad = WORKLOADS[args.config]
    if args.batch is not None:
        B = args.batch
    cfg = {"batch": B, "seq": S, "d_model": D, "heads": H, "ffn": F, "layers": L, "causal": causal}
    workload_name = args.config if args.batch is None else f"{args.config}-batch{B}"
    if args.impl == "reference":
        return run_reference(args, cfg, pad, workload_name)

    import torch.distributed as dist

    from tiktoktechjam2026_b200 import B200Transformer, TransformerConfig, _lib
    from tiktoktechjam2026_b200.model import default_host_chunk
    from tiktoktechjam2026_b200.sharding import PeerGatherBuffer, shard_bounds

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    strong = args.scaling == "strong"
    # Strong scaling (default): the workload's one batch of B sequences is split
    # into contiguous slices (shard_bounds), rank r runs sequences [s0, s1), and
    # every slice's FP32 output is pushed into one gather buffer on GPU 0 inside
    # the timed region.  Weak scaling: every rank runs a whole batch of B of its
    # own (seed SEED + r), nothing is gathered.
    if strong:
        s0, s1 = shard_bounds(B, world, rank)
        global_batch = B
    else:
        s0, s1 = 0, B
        global_batch = B * world
    nb = s1 - s0
    torch.manual_seed(1234)
    model = B200Transformer(TransformerConfig(nb, S, D, H, F, L, causal)).to(dev).eval()
    model.convert_projections_to_fp16()
    model.assume_all_tokens_valid = pad <= 0
    x_full, mask_full = make_inputs(cfg, pad, SEED if strong else SEED + rank)
    x_host = x_full[s0:s1].contiguous().pin_memory()
    mask_host = None if mask_full is None else mask_full[s0:s1].contiguous().pin_memory()
    x_all = x_full if (strong and world > 1 and rank == 0) else None  # for rank 0's 1-GPU check
    mask_all = mask_full if x_all is not None else None
    del x_full, mask_full
    x_dev = x_host.to(dev)
    mask_dev = None if mask_host is None else mask_host.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    gather = None
    outs = [torch.empty_like(x_dev) for _ in range(2)]
    if strong and world > 1:
        gather = PeerGatherBuffer(B, (S, D), rank, world, dev, slots=2)
        if rank == 0:
            outs = [gather.local_view(k)[s0:s1] for k in range(2)]

    def step(i):
        """One forward of this rank's slice; with a gather, its output pushed to GPU 0."""
        if gather is None:
            model.forward_gather(x_dev, mask_dev, outs[i % 2], 0)
        else:
            model.forward_gather(x_dev, mask_dev, outs[i % 2], gather.dst(i % 2) if rank != 0 else 0)

    def timed_steps(fn, n, tail=None):
        """Per-step CUDA-event times with the L2 flushed (untimed) before each step,
        plus the time `tail` adds after the last step; summed, in ms."""
        st = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        en = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        barrier()
        for i in range(n):
            flush.zero_()
            st[i].record(stream)
            fn(i)
            en[i].record(stream)
        st[n].record(stream)
        if tail is not None:
            tail()
        en[n].record(stream)
        barrier()
        return [a.elapsed_time(b) for a, b in zip(st, en)]

    with torch.inference_mode():
        for i in range(max(3, args.warmup)):
            step(i)
        if gather is not None:
            model.gather_wait(dev)
        barrier()

        # ---------------- value: device-resident inputs ----------------
        # --graph replays one captured forward per step (tt_model_graph_create);
        # the per-kernel breakdown then comes from a separate profiled eager pass.
        graphed = None
        kernels_per_forward = 0
        if args.graph and gather is None:
            l0 = _lib.lib().tt_launch_count()
            model(x_dev, mask_dev)
            kernels_per_forward = _lib.lib().tt_launch_count() - l0
            graphed = model.capture_graph(x_dev, mask_dev)
            for _ in range(3):
                graphed()
            barrier()
        sampler = ClockSampler() if rank == 0 else None
        if sampler:
            sampler.start()
        launches0 = _lib.lib().tt_launch_count()
        if graphed is not None:
            step_ms = timed_steps(lambda i: graphed(), args.steps)
        else:
            step_ms = timed_steps(step, args.steps, (lambda: model.gather_wait(dev)) if gather is not None else None)
        launches = _lib.lib().tt_launch_count() - launches0 + kernels_per_forward * args.steps
        # Per-kernel breakdown from a separate profiled pass of the same steps: the
        # library's events around every launch would keep consecutive kernels from
        # overlapping their set-up (programmatic dependent launch) in the timed steps.
        model.set_profiling(True, dev)
        model.profile_collect(dev)
        prof_step_ms = timed_steps(lambda i: model.forward_gather(x_dev, mask_dev, outs[i % 2], 0), args.steps)
        prof = model.profile_collect(dev)
        model.set_profiling(False, dev)
        total_ms = max_over_ranks(sum(step_ms))
        gather_tail_ms = max_over_ranks(step_ms[-1])

        extra = {}
        if world > 1:
            # Each rank's own ms per step, to see which one sets the max.
            mine = torch.tensor([sum(step_ms) / args.steps, float(nb)], dtype=torch.float64, device=dev)
            every = [torch.zeros_like(mine) for _ in range(world)]
            dist.all_gather(every, mine)
            extra["rank_ms_per_step"] = [round(float(t[0]), 4) for t in every]
            extra["rank_sequences"] = [int(t[1]) for t in every]
        if gather is not None:
            # Compute alone (no push), and one step's latency with the push exposed.
            comp = timed_steps(lambda i: model.forward_gather(x_dev, mask_dev, outs[i % 2], 0), args.steps)
            extra["compute_only"] = {"value": global_batch * 1000.0 / (max_over_ranks(sum(comp)) / args.steps),
                                     "ms_per_step": max_over_ranks(sum(comp)) / args.steps,
                                     "what": "the same steps without the push to GPU 0"}
            lat = []
            for i in range(args.steps):
                t = timed_steps(lambda j: (step(i), model.gather_wait(dev)), 1)
                lat.append(max_over_ranks(sum(t)))
            extra["latency_ms"] = {"median": statistics.median(lat), "max": max(lat),
                                   "what": "one step alone: slice forward, then its push to GPU 0 waited for"}
            # Rank 0 checks the gathered batch against its own 1-GPU forward of the whole batch.
            barrier()
            if rank == 0:
                full_model = model
                ref = full_model(x_all.to(dev), None if mask_all is None else mask_all.to(dev))
                torch.cuda.synchronize(dev)
                got = gather.local_view((args.steps - 1) % 2)
                extra["gather_check"] = {
                    "sequences": B, "bitwise_equal_to_1gpu_forward": bool(torch.equal(got, ref)),
                    "max_abs_diff": float((got - ref).abs().max().item())}
                del ref
            barrier()
            # Weak scaling for comparison: every rank runs a whole batch of its own.
            xw, mw = make_inputs(cfg, pad, SEED + rank)
            xw = xw.to(dev)
            mw = None if mw is None else mw.to(dev)
            ow = torch.empty_like(xw)
            model(xw, mw)
            weak = timed_steps(lambda i: model.forward_gather(xw, mw, ow, 0), args.steps)
            extra["weak"] = {"value": B * world * 1000.0 / (max_over_ranks(sum(weak)) / args.steps),
                             "ms_per_step": max_over_ranks(sum(weak)) / args.steps, "global_batch": B * world,
                             "what": f"each rank runs a whole batch of {B} of its own; nothing gathered"}
            del xw, mw, ow

        # ---------------- e2e: host buffers through the public call ----------------
        # model.forward_host = one tt_model_forward_host call: pinned host input in,
        # pinned host output back, copies pipelined with the kernels by chunks.  With
        # several ranks each writes its slice into one host buffer shared with rank 0.
        chunk = args.chunk or default_host_chunk(nb, S, D)
        host_out = SharedHostOutput((B, S, D), s0, s1, rank, world, barrier) if strong and world > 1 else None
        out_host = host_out.part if host_out is not None else torch.empty_like(x_host).pin_memory()
        for _ in range(2):
            model.forward_host(x_host, mask_host, out=out_host, chunk=chunk)
        barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        barrier()
        e_start.record(stream)
        for _ in range(args.steps):
            model.forward_host(x_host, mask_host, out=out_host, chunk=chunk)
        e_end.record(stream)
        barrier()
        clocks = sampler.stop(list(range(world))) if sampler else None
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end))
        if host_out is not None:
            if rank == 0 and host_out.all_shared:
                ref = model(x_all.to(dev), None if mask_all is None else mask_all.to(dev)).cpu()
                extra["e2e_gather_check"] = {"sequences": B,
                                             "bitwise_equal_to_1gpu_forward": bool(torch.equal(host_out.full, ref))}
                del ref
            extra["e2e_gather"] = ("one host buffer shared by all ranks (/dev/shm, page-locked per slice)"
                                   if host_out.all_shared else "per-rank pinned buffers (no shared host memory)")
            host_out.close(rank, barrier)

    # ---------------- roofline of the dominant kernel ----------------
    hbm_peak, tc_peak, peak_src = load_peaks()
    dominant = max(((k, v) for k, v in prof.items() if v[1] > 0), key=lambda kv: kv[1][0])
    kind, (kms, kcount) = dominant
    per_launch_s = kms / kcount / 1e3
    flops, nbytes = algorithmic(cfg, nb)[kind]
    t_tc = flops / (tc_peak * 1e12)
    t_hbm = nbytes / (hbm_peak * 1e9)
    if t_tc >= t_hbm:
        roof = {"bound": "tensor", "achieved": flops / per_launch_s / 1e12, "peak": tc_peak, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": nbytes / per_launch_s / 1e9, "peak": hbm_peak, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = load_traffic(args.config if args.batch is None else workload_name, nb, kind)
    roof["kernel"] = kernel_label(kind, cfg)
    roof["mean_launch_us"] = per_launch_s * 1e6
    roof["algorithmic_per_launch"] = {"flops": flops, "bytes": nbytes}
    roof["peak_source"] = f"{peak_src} ({'bf16_tflops burst' if roof['bound'] == 'tensor' else 'hbm_gbs'})"
    roof["share_of_step"] = kms / max(sum(prof_step_ms), 1e-9)
    roof["measured_over"] = (f"a profiled pass of the same {args.steps} steps after the timed ones "
                             f"({sum(prof_step_ms) / args.steps:.3f} ms per step with the events)")

    if rank == 0:
        ms_per_step = total_ms / args.steps
        value = global_batch * 1000.0 / ms_per_step
        e2e_value = global_batch * 1000.0 / (e2e_ms / args.steps)
        if strong:
            par = (f"batch split x{world}: {nb} sequences on GPU 0 (shard_bounds), FP32 outputs pushed into one "
                   f"gather buffer on GPU 0 over NVLink (copy engines, overlapped with the next step)"
                   if world > 1 else "one GPU, whole batch")
        else:
            par = f"weak scaling x{world}: {nb} sequences per GPU, no collective in the data path"
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "f16 tensor-core operands, f32 accumulate/softmax/LayerNorm/residual",
            "data": "synthetic (x ~ N(0,1) FP32 from the reference's timing seed; seeded default-init weights)",
            "config": {"workload": f"{workload_name}: batch {B}, seq {S}, d_model {D}, heads {H}, ffn {F}, "
                                   f"layers {L}, causal{', key padding' if pad > 0 else ''}",
                       "global_batch": global_batch, "per_gpu_batch": nb, "seq_len": S, "d_model": D, "heads": H,
                       "ffn": F, "layers": L, "parallelism": par,
                       "l2": "flushed between timed steps (256 MiB write, untimed)",
                       "launch": "one CUDA graph replay per step" if graphed is not None else
                                 "eager (one host call per step)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": e2e_ms / args.steps, "chunk": chunk,
                    "path": "model.forward_host -> tt_model_forward_host (pinned host in/out, copies overlapped "
                            "with compute by chunks)" + ("; each rank's slice of one shared host output" if
                                                         strong and world > 1 else ""),
                    "h2d_bytes_per_step": (world if not strong else 1) * (
                        B * S * D * 4 + (0 if mask_host is None else B * S)),
                    "d2h_bytes_per_step": (world if not strong else 1) * B * S * D * 4},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernel_ms_per_step": {k: v[0] / args.steps for k, v in prof.items() if v[1] > 0},
            "clocks": clocks,
        }
        if gather is not None:
            line["gather"] = {"bytes_into_gpu0_per_step": (B - nb) * S * D * 4,
                              "tail_ms": gather_tail_ms,
                              "what": "each step's push overlaps the next step's compute; tail_ms is the wait "
                                      "for the last push after the last step, inside the timed total"}
        line.update(extra)
        if world == 1 and not args.no_cpu_baseline:
            v, cores, sample = cpu_baseline(cfg, pad, args.cpu_sample_seconds)
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
        print(json.dumps(line), flush=True)
    if gather is not None:
        barrier()
        gather.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
