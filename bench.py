"""Benchmark: 7B-shape batched greedy decode on B200 (sm_100a kernels).

Workload (the decode config): Llama-2-7B shape (32 layers, hidden 4096,
32 heads x 128, FFN 11008, vocab 32000), random-init bf16 weights ~N(0, 0.02)
with RMSNorm weights 1.0, 256 prompts of 512 tokens drawn uniformly over the
vocabulary (seed 3), greedy decode.  The 256 sequences are split in
contiguous chunks over the ranks (256/128/64/32 per GPU at 1/2/4/8 GPUs), one
process per GPU, full weight replica each, no collective on the data path.

A "step" is one batched decode step of the whole model for the rank's
sequences (embedding -> 32 layers -> norm -> lm_head -> argmax), replayed from
one CUDA graph.  Untimed steps run first so that the timed steps are centred
on the mean context of a 128-token generation (prompt + 64).  Every step
reads ~90 GB (weights + KV cache) at N=1, far more than L2: no flush needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU oracle port
of the reference's PyTorch path on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "7B-shape decode tok/s at 1/2/4/8 B200; per-kernel % of HBM / TC roofline"
UNIT = "tok/s"
GLOBAL_BATCH = 256
PROMPT_LEN = 512
NEW_TOKENS = 128
SEED = 3
# ncu dram bytes (read + write) / algorithmic bytes of the decode-attention
# kernel, from one full capture of the split kernel on one layer of the decode
# config (256 sequences at 576 keys: 2,418.0 MB read + 6.0 MB written for
# 2,420.1 MB of K/V, q and output).  The bench scales it to its own launch
# (traffic grows with the K/V bytes processed).
DECODE_ATTN_TRAFFIC_RATIO = (2418.039e6 + 5.953536e6) / 2420.113408e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH)
    ap.add_argument("--prompt-len", type=int, default=PROMPT_LEN)
    ap.add_argument("--layers", type=int, default=32, help="(debug only) fewer layers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pre-steps", type=int, default=None,
                    help="untimed decode steps before the timed ones (default: enough to centre "
                         "the timed steps on the mean context)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--suite", choices=["decode", "ops", "longctx", "kernels"], default="decode",
                    help="decode: the 7B decode workload (default); ops: per-op roofline lines; "
                         "longctx: 64 prompts of 1k-8k tokens, prefill + 256 decode steps; "
                         "kernels: the per-kernel roofline entries of the decode line")
    ap.add_argument("--only", default="", help="comma list of op lines for --suite ops, or of "
                    "kernel keys for --suite kernels (" + ", ".join(KERNEL_KEYS) + ")")
    ap.add_argument("--no-kernels", action="store_true",
                    help="skip the per-kernel roofline block of the decode line")
    ap.add_argument("--no-longctx", action="store_true",
                    help="skip the long-context block of the decode line")
    ap.add_argument("--decode-batch", type=int, default=64,
                    help="sequences of the ragged decode op line (64 = the decode op shape)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        under = [s for s in sm if s > 0.5 * (max(smax) if smax else 1)] or sm
        return {"sm_mhz": statistics.median(under) if under else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def smi_index(local: int) -> int:
    """nvidia-smi index of this process's GPU (CUDA_VISIBLE_DEVICES remaps it)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            pass
    return local


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def shard(global_batch: int, world: int, rank: int):
    """Contiguous chunk of sequences for this rank (256/N each)."""
    per = global_batch // world
    extra = global_batch % world
    start = rank * per + min(rank, extra)
    return start, per + (1 if rank < extra else 0)


def _coll_device():
    import torch.distributed as dist
    return "cpu" if dist.get_backend() == "gloo" else "cuda"


def max_over_ranks(x: float, world: int) -> float:
    """Max of a per-rank scalar (timings are reported as the slowest rank)."""
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=_coll_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        t = torch.zeros(1, device=_coll_device())
        dist.all_reduce(t)
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def model_config(layers: int, max_seq: int):
    from llama_pure_compute_b200.config import PRESETS, LlamaModelConfig
    base = PRESETS["llama-2-7b"]
    return LlamaModelConfig(vocab_size=base.vocab_size, dim=base.dim, inter_dim=base.inter_dim,
                            num_layers=layers, num_heads=base.num_heads,
                            num_kv_heads=base.num_kv_heads, max_seq_len=max_seq,
                            rms_norm_eps=1e-5, rope_theta=10000.0)


def prompts_for(rank_start: int, count: int, prompt_len: int, global_batch: int):
    g = torch.Generator().manual_seed(SEED)
    allp = torch.randint(0, 32000, (global_batch, prompt_len), generator=g)
    return allp[rank_start:rank_start + count]


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference's PyTorch CPU path
# ---------------------------------------------------------------------------
def cpu_decode_baseline(layers: int, seconds: float, batch: int = 4, ctx: int = 576):
    """Times decode steps of the 7B shape on the host cores with the CPU oracle
    (fp32 torch on CPU).  Bounded sample: `batch` sequences with a random
    `ctx`-token KV cache, as many steps as fit in ~`seconds`; the 32 layers
    share one layer's random weights (same arithmetic and per-layer weight
    bytes; keeps host memory and set-up time small)."""
    from oracle.model_ref import OracleLlama
    torch.manual_seed(SEED)
    cfg = dict(vocab_size=32000, dim=4096, inter_dim=11008, num_layers=layers, num_heads=32,
               num_kv_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0)
    D, I, V = 4096, 11008, 32000
    layer = {
        "input_layernorm.weight": torch.ones(D),
        "self_attn.q_proj.weight": torch.randn(D, D) * 0.02,
        "self_attn.k_proj.weight": torch.randn(D, D) * 0.02,
        "self_attn.v_proj.weight": torch.randn(D, D) * 0.02,
        "self_attn.o_proj.weight": torch.randn(D, D) * 0.02,
        "post_attention_layernorm.weight": torch.ones(D),
        "gate_proj.weight": torch.randn(I, D) * 0.02,
        "up_proj.weight": torch.randn(I, D) * 0.02,
        "down_proj.weight": torch.randn(D, I) * 0.02,
    }
    sd = {"model.embed_tokens.weight": torch.randn(V, D) * 0.02, "model.norm.weight": torch.ones(D),
          "lm_head.weight": torch.randn(V, D) * 0.02}
    for i in range(layers):
        for k, v in layer.items():
            sd[f"model.layers.{i}.{k}"] = v
    orc = OracleLlama(cfg, sd, max_seq_len=ctx + 256)
    cache = [[torch.randn(batch, 32, ctx, 128), torch.randn(batch, 32, ctx, 128)]
             for _ in range(layers)]
    tok = torch.randint(0, V, (batch, 1))
    times = []
    t_end = time.perf_counter() + seconds
    pos = ctx
    with torch.no_grad():
        while True:
            t0 = time.perf_counter()
            logits = orc.forward(tok, torch.full((batch, 1), pos), cache)
            tok = logits[:, -1].argmax(-1, keepdim=True)
            times.append(time.perf_counter() - t0)
            pos += 1
            if time.perf_counter() > t_end and len(times) >= 2:
                break
    steady = times[1:] if len(times) > 1 else times
    sec = statistics.median(steady)
    return {"value": batch / sec, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": (f"CPU oracle (fp32 torch on host, {torch.get_num_threads()} threads): "
                       f"{len(times)} decode steps of {batch} sequences at context {ctx}..{pos - 1}, "
                       f"{layers} layers sharing one layer's random weights; median step "
                       f"{sec * 1e3:.1f} ms")}


def run_reference(args, world, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    cb = cpu_decode_baseline(args.layers, args.cpu_seconds * max(1, args.steps) / 20.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(cb["value"], 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(4 / cb["value"] * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama-2-7b batched greedy decode (bounded CPU sample)",
                   "global_batch": GLOBAL_BATCH, "prompt_len": args.prompt_len,
                   "new_tokens": NEW_TOKENS},
        "cpu_baseline": cb,
        "e2e": {"value": round(cb["value"], 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU run
# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    from llama_pure_compute_b200 import _lib
    from llama_pure_compute_b200.generate import BatchedGreedyDecoder
    from llama_pure_compute_b200.kv_manager import KVCacheManager
    from llama_pure_compute_b200.model import LlamaForCausalLM
    from llama_pure_compute_b200.ops import decode_attention

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _lib.load()
    start, count = shard(args.batch, world, rank)
    mean_ctx = args.prompt_len + NEW_TOKENS // 2
    pre_steps = max(args.warmup, mean_ctx - args.prompt_len - args.steps // 2)
    if args.pre_steps is not None:
        pre_steps = max(args.warmup, args.pre_steps)
    max_seq = args.prompt_len + max(NEW_TOKENS, pre_steps + args.steps + 2)
    cfg = model_config(args.layers, max_seq)

    model = LlamaForCausalLM.random_init(cfg, device=dev, dtype=torch.bfloat16, seed=SEED)
    kv = KVCacheManager(num_layers=cfg.num_layers, max_batch_size=count, max_seq_len=max_seq,
                        n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, dtype=torch.bfloat16,
                        device=dev)
    prompts = prompts_for(start, count, args.prompt_len, args.batch)
    dec = BatchedGreedyDecoder(model, kv, count, use_cuda_graph=True)

    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    dec.prefill(prompts)
    t1.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(t0.elapsed_time(t1), world)

    n0 = _lib.launch_count
    dec.capture()  # runs the step body twice: one eager warm-up, one captured
    launches_per_step = (_lib.launch_count - n0) // 2

    clocks = ClockSampler(smi_index(local))
    clocks.start()
    for _ in range(pre_steps):  # untimed warm-up steps (also move to the mean context)
        dec.step()
    barrier(world)
    ctx_first = int(dec.positions[0, 0].item())
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        dec.step()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, world)
    tok_s = args.batch * args.steps / (ms_max / 1e3)

    # ---- e2e: public API, host token buffers, H2D + D2H inside every step ----
    # Every step copies its tokens and positions from pinned host memory and
    # its result (the next tokens) back into pinned host memory.  The token
    # round trip goes through one pinned buffer in stream order (the result's
    # D2H, then the next step's H2D), so the host never stalls the device; it
    # reads each step's result from the pinned results array as the step
    # completes, one step behind the device.
    B = count
    e_steps = max(2, min(args.steps, 20))
    host_tok = torch.empty(B, dtype=torch.long, pin_memory=True)
    host_pos = torch.empty(e_steps, B, dtype=torch.long, pin_memory=True)
    host_res = torch.empty(e_steps, B, dtype=torch.long, pin_memory=True)
    host_tok.copy_(dec.tokens[:, 0].cpu())
    # the same contexts as the device-timed steps (their cache rows are rewritten)
    pos0 = dec.positions[:, 0].cpu() - args.steps
    host_pos.copy_(pos0.unsqueeze(0) + torch.arange(e_steps).unsqueeze(1))
    done = [torch.cuda.Event() for _ in range(e_steps)]
    seen = 0
    barrier(world)
    w0 = time.perf_counter()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(e_steps):
        dec.tokens[:, 0].copy_(host_tok, non_blocking=True)
        dec.positions[:, 0].copy_(host_pos[i], non_blocking=True)
        out = dec.step()
        host_res[i].copy_(out, non_blocking=True)
        host_tok.copy_(out, non_blocking=True)  # the next step's input, in stream order
        done[i].record()
        if i > 0:  # the host consumes the previous step's result while this one runs
            done[i - 1].synchronize()
            seen += int(host_res[i - 1].min() >= 0)
    s1.record()
    torch.cuda.synchronize()
    seen += int(host_res[e_steps - 1].min() >= 0)
    assert seen == e_steps, "e2e: a step's result did not reach the host"
    e2e_ms = max_over_ranks(s0.elapsed_time(s1), world)
    wall_e2e = max_over_ranks((time.perf_counter() - w0) * 1e3, world)
    e2e_tok_s = args.batch * e_steps / (e2e_ms / 1e3)
    clk = clocks.stop()
    # device-side error flags (bounded waits that gave up, bounds checks) of
    # every kernel run so far: a run with any flag set is not a measurement
    status = int(max_over_ranks(float(_lib.device_status()), world))

    # ---- dominant kernel: split-KV decode attention, timed standalone on the
    # final decode state (layer 0 cache, current per-sequence lengths) ----
    lens = kv.seq_lens[:B].clone()
    q = torch.randn(B, cfg.num_heads, cfg.head_dim, device=dev, dtype=torch.bfloat16)
    ws = kv.decode_workspace(B, cfg.num_heads)
    outb = torch.empty_like(q)
    for _ in range(3):
        decode_attention(q, kv.k_cache[0], kv.v_cache[0], lens, None, outb, ws)
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    reps = 10
    # a GPU-side sleep queued first keeps the host's launches ahead of the
    # device, so the timed launches run back to back as they do in the step's
    # graph (at 32 sequences a call is ~50 us, near the host's launch cost)
    torch.cuda._sleep(2_000_000)
    a0.record()
    for i in range(reps):
        decode_attention(q, kv.k_cache[i % cfg.num_layers], kv.v_cache[i % cfg.num_layers], lens,
                         None, outb, ws)
    a1.record()
    torch.cuda.synchronize()
    attn_us = a0.elapsed_time(a1) * 1e3 / reps
    ctx_sum = int(lens.sum().item())
    attn_bytes = ctx_sum * cfg.num_kv_heads * cfg.head_dim * 2 * 2 + 2 * B * cfg.num_heads * cfg.head_dim * 2
    attn_gbs = attn_bytes / (attn_us * 1e-6) / 1e9
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    read_peak = measure_read_peak(dev)
    # algorithmic bytes of one decode step: every weight once (the embedding
    # table only for the B gathered rows) + the KV cache at the timed steps'
    # mean context
    emb = model.model.embed_tokens.weight
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    weight_bytes += (B - emb.shape[0]) * emb.shape[1] * emb.element_size()
    mean_ctx_timed = ctx_first + (args.steps + 1) / 2
    kv_bytes = int(B * mean_ctx_timed) * cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    step_bytes = weight_bytes + kv_bytes
    n_layers = cfg.num_layers
    dec.release()
    del dec, model, kv, q, outb, ws
    torch.cuda.empty_cache()

    kernels = None
    if not args.no_kernels:
        kernels = measure_kernels(dev)
        status = max(status, int(max_over_ranks(float(_lib.device_status()), world)))
    longctx = None
    if not args.no_longctx and args.layers == 32:
        torch.cuda.empty_cache()
        longctx = longctx_measure(args, world, rank, local)
        status = max(status, int(longctx.get("device_status", 0)))

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            cpu = cpu_decode_baseline(args.layers, args.cpu_seconds)
        line = {
            "metric": METRIC,
            "value": round(tok_s, 1),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "pre_steps": pre_steps,
            "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": {
                "workload": "llama-2-7b batched greedy decode, 256 prompts x 512 tokens, "
                            "steps timed around mean context 576",
                "model": "llama-2-7b shape (32L, 4096, 32x128 heads, FFN 11008, vocab 32000)",
                "global_batch": args.batch,
                "per_gpu_batch": count,
                "seq_len": args.prompt_len,
                "context_timed": [ctx_first, ctx_first + args.steps - 1],
                "parallelism": f"sequence-sharded replicas x{world} (no collective)",
                "l2": "inputs larger than L2 (each step streams ~13 GB weights + KV cache)",
                "layers": n_layers,
                "pre_steps": "untimed decode steps before the timed ones (the first `warmup` of "
                             "them are the warm-up; all move the context to the timed window)",
            },
            "clocks": clk,
            "e2e": {"value": round(e2e_tok_s, 1), "unit": UNIT, "h2d_bytes_per_step": 2 * 8 * B,
                    "d2h_bytes_per_step": 2 * 8 * B, "steps": e_steps,
                    "wall_ms": round(wall_e2e, 2)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {
                "kernel": "decode_split_kernel (+ decode_combine_kernel when a split does not "
                          "cover the cache length): split-KV decode attention",
                "bound": "hbm",
                "achieved": round(attn_gbs, 1),
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": round(attn_gbs / hbm_peak, 4),
                "traffic": int(attn_bytes * DECODE_ATTN_TRAFFIC_RATIO),
                "traffic_source": "ncu dram__bytes of the split kernel on one layer of this "
                                  "workload (256 sequences at 576 keys), scaled by the K/V "
                                  "bytes of this launch",
                "algorithmic_bytes_per_launch": attn_bytes,
                "launch_us": round(attn_us, 2),
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (burst)" if peaks else "fallback 6650",
                "read_peak": round(read_peak, 1),
                "frac_of_read_peak": round(attn_gbs / read_peak, 4),
                "read_peak_source": "lpc_hbm_read_probe on 4 GiB in this run: a read-only stream "
                                    "of 128 KB bulk-copy items (the peak above is a copy, which "
                                    "moves every byte twice)",
            },
            "step_roofline": {
                "bytes_per_step": step_bytes,
                "achieved_gbs": round(step_bytes / (ms_max / args.steps * 1e-3) / 1e9, 1),
                "frac": round(step_bytes / (ms_max / args.steps * 1e-3) / 1e9 / hbm_peak, 4),
            },
            "prefill": {"tokens": args.batch * args.prompt_len,
                        "ms": round(prefill_ms, 1),
                        "tok_s": round(args.batch * args.prompt_len / (prefill_ms / 1e3), 1)},
            "cpu_baseline": cpu,
            "device_status": status,
            "kernels": kernels,
            "longctx": longctx,
        }
        print(json.dumps(line), flush=True)
    if status:
        print(f"device status {status:#x}: a kernel flagged a timeout or a bounds failure; "
              "the numbers above are not valid", file=sys.stderr, flush=True)
        raise SystemExit(3)


def measure_read_peak(dev, nbytes: int = 4 << 30, reps: int = 10) -> float:
    """HBM read ceiling in GB/s: lpc_hbm_read_probe over a buffer far larger
    than L2, launched back to back and timed with CUDA events."""
    from llama_pure_compute_b200 import _lib
    lib = _lib.load()
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(3):
        _lib.check(lib.lpc_hbm_read_probe(buf.data_ptr(), nbytes, st), "hbm_read_probe")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(reps):
        lib.lpc_hbm_read_probe(buf.data_ptr(), nbytes, st)
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / reps
    del buf
    return nbytes / (us * 1e-6) / 1e9


# ---------------------------------------------------------------------------
# per-kernel rooflines in the decode line (same run, CUDA events)
# ---------------------------------------------------------------------------
def _kentry(kernel, shape, us, *, nbytes=None, flops=None, hbm, tc, timing):
    d = {"kernel": kernel, "shape": shape, "us": round(us, 2), "timing": timing}
    if nbytes is not None:
        d["bytes"] = int(nbytes)
        d["achieved_gbs"] = round(nbytes / us / 1e3, 1)
        d["frac_hbm"] = round(nbytes / us / 1e3 / hbm, 4)
    if flops is not None:
        d["flops"] = int(flops)
        d["tflops"] = round(flops / us / 1e6, 1)
        d["frac_tc"] = round(flops / us / 1e6 / tc, 4)
    return d


KERNEL_KEYS = ("swiglu_pair", "wsgemm_swiglu", "wsgemm_qkv", "wsgemm_resid", "prefill", "swiglu_f32",
               "rope_kv_append", "kv_append", "rmsnorm", "decode", "decode_b256")


def measure_kernels(dev, only=None):
    """Device time of each hot-path kernel at its benchmark shape, with the
    algorithmic bytes / FLOPs of one launch and the fraction of the measured
    peaks (HBM copy GB/s; dense bf16 TF/s, burst).  Weight-streaming kernels are
    timed in steady state, launches back to back over distinct weights whose
    total exceeds L2 (what a decode step does); the others over inputs larger
    than L2, or rotated over several input sets whose total exceeds it.
    ``only``: a set of KERNEL_KEYS to measure (all by default)."""
    from llama_pure_compute_b200 import ops
    from llama_pure_compute_b200.flash_attention import flash_attention_v2
    from llama_pure_compute_b200.model import precompute_freqs_cis
    from llama_pure_compute_b200.packed_linear import PackedWeight, packed_linear
    pk = _peaks()
    hbm = pk.get("hbm_gbs", 6650.0)
    tc = pk.get("bf16_tflops", 1590.0)
    bf = torch.bfloat16
    D, I, H = 4096, 11008, 32
    out = []
    steady = "steady state: back to back over distinct weight sets (> L2)"
    rot = "back to back over distinct input sets (> L2 in total)"
    g = torch.Generator(device=dev).manual_seed(5)

    def rn(*shape, std=1.0, dtype=bf):
        return (std * torch.randn(*shape, device=dev, generator=g)).to(dtype)

    want = lambda key: not only or key in only  # noqa: E731
    w1 = torch.ones(D, device=dev, dtype=bf)
    M = 32
    B, S = 4, 2048
    with torch.inference_mode():
        if want("swiglu_pair") or want("wsgemm_swiglu"):
            ws = [rn(2 * I, D, std=0.02) for _ in range(6)]
        if want("swiglu_pair"):
            # SwiGLU of the 7B layer at 256 tokens: row norm + CTA-pair tcgen05
            # GEMM launched under it (the decode step's path), and the one-kernel
            # form with the norm inside (norm weight folded into gate/up)
            M = 256
            x = rn(M, D)
            empty = torch.empty(0, device=dev, dtype=bf)
            us = _time_rotating([lambda w=w: ops.rmsswiglu_forward(x, w1, w, empty, 1e-5)
                                 for w in ws])
            out.append(_kentry("rmsnorm_vec_kernel + swiglu_pair_kernel", "7B gate/up, 256 tokens",
                               us, nbytes=2 * I * D * 2 + M * D * 2 + M * I * 2,
                               flops=2 * M * D * 2 * I, hbm=hbm, tc=tc, timing=steady))
            us = _time_rotating([lambda w=w: ops.rmsswiglu_folded_forward(x, w, None, 1e-5)
                                 for w in ws])
            out.append(_kentry("swiglu_pair_kernel (norm inside)", "7B gate/up, 256 tokens", us,
                               nbytes=2 * I * D * 2 + M * D * 2 + M * I * 2,
                               flops=2 * M * D * 2 * I, hbm=hbm, tc=tc, timing=steady))
        if want("wsgemm_swiglu"):
            # decode-sized norm + SwiGLU on packed weights (32 tokens): the
            # decode step's form, the norm weight folded into the packed copy
            nw = 1 + 0.02 * rn(D)
            pws = [PackedWeight(w, layout="swiglu", norm_weight=nw) for w in ws]
            M = 32
            x = rn(M, D)
            us = _time_rotating([lambda pw=pw: packed_linear(x, pw, "swiglu", norm_eps=1e-5)
                                 for pw in pws])
            out.append(_kentry("wsgemm_kernel (norm + SwiGLU epilogue)", "7B gate/up, 32 tokens",
                               us, nbytes=2 * I * D * 2 + M * D * 2 + M * I * 2, hbm=hbm, tc=tc,
                               timing=steady))
            del pws
        if want("swiglu_pair") or want("wsgemm_swiglu"):
            del ws
        if want("wsgemm_qkv"):
            # q/k/v projection + RoPE + KV append (32 tokens, normed input)
            M = 32
            wq = [rn(3 * H * 128, D, std=0.02) for _ in range(6)]
            nq = 1 + 0.02 * rn(D)
            pq = [PackedWeight(w, layout="heads", norm_weight=nq) for w in wq]
            cos, sin = precompute_freqs_cis(128, 1024, device=dev)
            cos, sin = cos.to(bf), sin.to(bf)
            x = rn(M, 1, D)
            pos = torch.randint(0, 1000, (M, 1), device=dev, generator=g)
            kc = torch.zeros(M, H, 1024, 128, device=dev, dtype=bf)
            vc = torch.zeros_like(kc)
            us = _time_rotating([lambda pw=pw: ops.qkv_rope_append(x, pw, pos, cos, sin, kc, vc, H,
                                                                   H, norm_eps=1e-5) for pw in pq])
            out.append(_kentry("wsgemm_kernel (EPI_QKV: norm + projection + RoPE + KV append)",
                               "7B q/k/v, 32 tokens", us,
                               nbytes=3 * H * 128 * D * 2 + M * D * 2 + M * 3 * H * 128 * 2,
                               hbm=hbm, tc=tc, timing=steady))
            del wq, pq, kc, vc
        if want("wsgemm_resid"):
            # o_proj and down_proj + residual on packed weights (32 tokens)
            M = 32
            po = [PackedWeight(rn(D, D, std=0.02)) for _ in range(12)]
            pd = [PackedWeight(rn(D, I, std=0.02)) for _ in range(6)]
            xo, xd, r = rn(M, D), rn(M, I), rn(M, D)
            for name, pws, xin, kin in (("o_proj", po, xo, D), ("down_proj", pd, xd, I)):
                us = _time_rotating([lambda pw=pw: packed_linear(xin, pw, "residual", resid=r, out=r)
                                     for pw in pws])
                out.append(_kentry("wsgemm_kernel (residual epilogue, split k)",
                                   f"7B {name}, 32 tokens", us,
                                   nbytes=D * kin * 2 + M * kin * 2 + 2 * M * D * 2, hbm=hbm, tc=tc,
                                   timing=steady))
            del po, pd
        if want("prefill"):
            # prefill attention [4, 32, 2048, 128] causal
            q, k, v = (rn(4, 32, 2048, 128) for _ in range(3))
            us = _time_us(lambda: flash_attention_v2(q, k, v, causal=True, sm_scale=128 ** -0.5), 10)
            out.append(_kentry("flash_prefill_kernel", "[4, 32, 2048, 128] causal", us,
                               nbytes=4 * 4 * 32 * 2048 * 128 * 2,
                               flops=2 * 4 * 32 * 2048 * 2048 * 128, hbm=hbm, tc=tc,
                               timing="inputs 201 MB (> L2), launches back to back"))
            del q, k, v
        if want("swiglu_f32"):
            # fp32 RMSNorm + SwiGLU op shape (x [8, 4096], W 2 x [11008, 4096] fp32)
            xf = rn(8, D, dtype=torch.float32)
            wf = 1 + 0.02 * torch.randn(D, device=dev, generator=g)
            gu = [(rn(I, D, std=0.02, dtype=torch.float32), rn(I, D, std=0.02, dtype=torch.float32))
                  for _ in range(2)]
            us = _time_rotating([lambda a=a, b=b: ops.rmsswiglu_forward(xf, wf, a, b, 1e-6)
                                 for a, b in gu])
            out.append(_kentry("swiglu_f32_kernel", "fp32 op: x [8, 4096], W 2 x [11008, 4096]", us,
                               nbytes=(2 * I * D + 8 * D + D + 8 * I) * 4, hbm=hbm, tc=tc,
                               timing=steady))
            del gu
        if want("rope_kv_append") or want("kv_append"):
            # RoPE + KV append at a prefill size: 4 x 2048 tokens
            sets = []
            cos, sin = precompute_freqs_cis(128, S, device=dev)
            cos, sin = cos.to(bf), sin.to(bf)
            posp = torch.arange(S, device=dev).unsqueeze(0).expand(B, -1).contiguous()
            for _ in range(3):
                sets.append((rn(B, S, 3 * H * 128), torch.empty(B, H, S, 128, device=dev, dtype=bf),
                             torch.empty(B, H, S, 128, device=dev, dtype=bf),
                             torch.empty(B, H, S, 128, device=dev, dtype=bf),
                             rn(B * S, H, 128), rn(B * S, H, 128)))
        if want("rope_kv_append"):
            us = _time_rotating([lambda t=t: ops.rope_kv_append(t[0], posp, cos, sin, t[1], t[2], H,
                                                                H, q_out=t[3]) for t in sets])
            out.append(_kentry("rope_kv_append_kernel", "4 x 2048 tokens, 32 + 2 x 32 heads", us,
                               nbytes=2 * B * S * 3 * H * 128 * 2, hbm=hbm, tc=tc, timing=rot))
        if want("kv_append"):
            # KV append alone (update_kv_cache) at the same size
            us = _time_rotating([lambda t=t: ops.update_kv_cache(t[4], t[5], t[1], t[2])
                                 for t in sets])
            out.append(_kentry("kv_append_rows_kernel", "8192 tokens x 32 heads x 128 (K and V)", us,
                               nbytes=2 * 2 * B * S * H * 128 * 2, hbm=hbm, tc=tc, timing=rot))
        if want("rope_kv_append") or want("kv_append"):
            del sets
        if want("rmsnorm"):
            # row RMSNorm at 8192 x 4096
            xs = [rn(B * S, D) for _ in range(4)]
            us = _time_rotating([lambda t=t: ops.rmsnorm_forward(t, w1, 1e-5) for t in xs])
            out.append(_kentry("rmsnorm_warp_kernel", "8192 x 4096", us,
                               nbytes=2 * B * S * D * 2 + D * 2, hbm=hbm, tc=tc, timing=rot))
            del xs
    if want("decode"):
        with torch.inference_mode():
            # decode attention at the decode op shape: 64 sequences, L ~ U[128, 4096]
            torch.manual_seed(2)
            L = torch.randint(128, 4097, (64,))
            Smax = 4097
            kc = rn(64, H, Smax, 128)
            vc = rn(64, H, Smax, 128)
            qd = rn(64, H, 128)
            lens = (L + 1).to(torch.int32).to(dev)
            wsd = ops.decode_attention_workspace(64, H, Smax, 128, dev)
            od = torch.empty_like(qd)
            us = _time_us(lambda: ops.decode_attention(qd, kc, vc, lens, None, od, wsd), 10)
            out.append(_kentry("decode_split_kernel + decode_combine_kernel (1024-key splits)",
                               "64 sequences, L ~ U[128, 4096], 32 heads x 128", us,
                               nbytes=int((L + 1).sum()) * H * 128 * 2 * 2 + 2 * 64 * H * 128 * 2,
                               hbm=hbm, tc=tc, timing="4.3 GB cache (> L2), launches back to back"))
            del kc, vc
    if want("decode_b256"):
        with torch.inference_mode():
            # one layer of the decode config: 256 sequences at context 576 in
            # a 616-key cache (one 1024-key split per sequence and KV head:
            # the split kernel alone, no combine launch)
            B2, L2, Smax2 = 256, 576, 616
            kc = rn(B2, H, Smax2, 128)
            vc = rn(B2, H, Smax2, 128)
            qd = rn(B2, H, 128)
            lens = torch.full((B2,), L2, dtype=torch.int32, device=dev)
            wsd = ops.decode_attention_workspace(B2, H, Smax2, 128, dev)
            od = torch.empty_like(qd)
            f = lambda: ops.decode_attention(qd, kc, vc, lens, None, od, wsd)  # noqa: E731
            us = _time_rotating([f] * 10)
            out.append(_kentry("decode_split_kernel",
                               "256 sequences at 576 keys, 32 heads x 128 (one layer of the decode config)",
                               us, nbytes=B2 * L2 * H * 128 * 2 * 2 + 2 * B2 * H * 128 * 2,
                               hbm=hbm, tc=tc, timing="2.4 GB of K/V (> L2); 10 launches back to back "
                                                        "behind a GPU sleep, best of 5"))
            del kc, vc
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# per-op roofline lines (--suite ops)
# ---------------------------------------------------------------------------
def _peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def _time_us(fn, reps: int, flush=None, warm: int = 3) -> float:
    """Mean device time of fn() in microseconds: CUDA events on the current
    stream, `flush` (an L2-sized write) between launches when given; the
    flush is timed separately and subtracted."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    total = 0.0
    for _ in range(reps):
        if flush is not None:
            flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        b.synchronize()
        total += a.elapsed_time(b)
    return total / reps * 1e3


def _time_rotating(fns, reps: int = 5) -> float:
    """Per-launch device time (us) of launches back to back over distinct
    inputs: a GPU sleep queued first keeps the host ahead of the device, and
    the best of `reps` passes is reported."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        torch.cuda._sleep(2_000_000)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for f in fns:
            f()
        b.record()
        b.synchronize()
        best = min(best, a.elapsed_time(b) * 1e3 / len(fns))
    return best


def run_ops(args):
    from llama_pure_compute_b200 import ops
    from llama_pure_compute_b200.flash_attention import flash_attention_v2
    from llama_pure_compute_b200.model import precompute_freqs_cis
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk = _peaks()
    hbm = pk.get("hbm_gbs", 6650.0)
    tc = pk.get("bf16_tflops", 1590.0)
    src = "MEASURED_PEAKS.json" if pk else "fallback"
    scratch = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)  # > L2 (126 MB)
    flush = lambda: scratch.fill_(1)  # noqa: E731
    only = set(filter(None, args.only.split(",")))
    out = []

    def emit(d):
        d.setdefault("peak_source", src)
        out.append(d)
        print(json.dumps(d), flush=True)

    if not only or "rmsswiglu_f32" in only:
        torch.manual_seed(0)
        x = torch.randn(8, 4096, device=dev)
        w = 1 + 0.02 * torch.randn(4096, device=dev)
        gw = 0.02 * torch.randn(11008, 4096, device=dev)
        uw = 0.02 * torch.randn(11008, 4096, device=dev)
        us = _time_us(lambda: ops.rmsswiglu_forward(x, w, gw, uw, 1e-6), 20, flush)
        byt = (2 * 11008 * 4096 + 8 * 4096 + 4096 + 8 * 11008) * 4
        emit({"op": "rmsswiglu_fp32 x[8,4096] W 2x[11008,4096]", "kernel": "swiglu_f32_kernel",
              "us": round(us, 2), "bytes": byt, "achieved_gbs": round(byt / us / 1e3, 1),
              "peak_gbs": hbm, "frac": round(byt / us / 1e3 / hbm, 4), "bound": "hbm",
              "l2": "flushed between launches"})
        del gw, uw
    if not only or "rmsswiglu_bf16" in only:
        for M in (256, 128, 64, 32):
            g = torch.Generator(device=dev).manual_seed(M)
            x = torch.randn(M, 4096, device=dev, generator=g).to(torch.bfloat16)
            w = torch.ones(4096, device=dev, dtype=torch.bfloat16)
            gw = (0.02 * torch.randn(11008, 4096, device=dev, generator=g)).to(torch.bfloat16)
            uw = (0.02 * torch.randn(11008, 4096, device=dev, generator=g)).to(torch.bfloat16)
            us = _time_us(lambda: ops.rmsswiglu_forward(x, w, gw, uw, 1e-5), 20, flush)
            byt = (2 * 11008 * 4096 + M * 4096 * 2 + M * 11008) * 2
            fl = 2 * M * 4096 * 2 * 11008
            emit({"op": f"rmsswiglu_bf16 7B layer M={M}", "kernel": "rmsnorm_vec + swiglu_tc_kernel",
                  "us": round(us, 2), "bytes": byt, "achieved_gbs": round(byt / us / 1e3, 1),
                  "frac_hbm": round(byt / us / 1e3 / hbm, 4), "tflops": round(fl / us / 1e6, 1),
                  "frac_tc": round(fl / us / 1e6 / tc, 4), "l2": "flushed between launches"})
    if not only or "swiglu_packed" in only:
        from llama_pure_compute_b200.packed_linear import PackedWeight, packed_linear
        # decode-sized SwiGLU of the 7B layer on packed weights, timed in steady
        # state: launches back to back over 6 distinct weight sets (1.1 GB, far
        # more than L2), as the decode graph runs them
        D, I, R = 4096, 11008, 6
        g = torch.Generator(device=dev).manual_seed(7)
        ws = [(0.02 * torch.randn(2 * I, D, device=dev, generator=g)).to(torch.bfloat16)
              for _ in range(R)]
        pws = [PackedWeight(w, layout="swiglu") for w in ws]
        rw = torch.ones(D, device=dev, dtype=torch.bfloat16)
        empty = torch.empty(0, device=dev, dtype=torch.bfloat16)
        for M in (32, 64, 128):
            x = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
            us = _time_rotating([lambda pw=pw: packed_linear(x, pw, "swiglu") for pw in pws])
            us_op = _time_rotating([lambda w=w: ops.rmsswiglu_forward(x, rw, w, empty, 1e-5)
                                    for w in ws])
            byt = 2 * I * D * 2 + M * D * 2 + M * I * 2
            emit({"op": f"swiglu 7B layer M={M} on packed weights", "kernel": "wsgemm_kernel",
                  "us": round(us, 2), "bytes": byt, "achieved_gbs": round(byt / us / 1e3, 1),
                  "peak_gbs": hbm, "frac": round(byt / us / 1e3 / hbm, 4), "bound": "hbm",
                  "fused_op_us": round(us_op, 2),
                  "l2": "steady state over 6 weight sets (1.1 GB > L2)"})
        del ws, pws
    if not only or "qkv_fused" in only:
        from llama_pure_compute_b200.packed_linear import PackedWeight
        # the attention block's projection + RoPE + KV append (one kernel on the
        # packed q/k/v weight) against cuBLAS + lpc_rope_kv_append, steady state
        # over 6 weight sets (604 MB > L2)
        H = Hkv = 32
        D, dim, R = 128, 4096, 6
        g = torch.Generator(device=dev).manual_seed(11)
        ws = [(0.02 * torch.randn((H + 2 * Hkv) * D, dim, device=dev, generator=g)).to(torch.bfloat16)
              for _ in range(R)]
        pws = [PackedWeight(w, layout="heads") for w in ws]
        cos, sin = precompute_freqs_cis(D, 1024, device=dev)
        cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
        for M in (8, 16, 32):
            x = torch.randn(M, 1, dim, device=dev, generator=g).to(torch.bfloat16)
            pos = torch.randint(0, 1000, (M, 1), device=dev, generator=g)
            kc = torch.zeros(M, Hkv, 1024, D, device=dev, dtype=torch.bfloat16)
            vc = torch.zeros_like(kc)
            us = _time_rotating([lambda pw=pw: ops.qkv_rope_append(x, pw, pos, cos, sin, kc, vc, H, Hkv)
                                 for pw in pws])
            us_two = _time_rotating([lambda w=w: ops.rope_kv_append(
                torch.mm(x.view(M, dim), w.t()).view(M, 1, -1), pos, cos, sin, kc, vc, H, Hkv)
                for w in ws])
            byt = (H + 2 * Hkv) * D * dim * 2 + M * dim * 2 + M * (H + 2 * Hkv) * D * 2
            emit({"op": f"qkv projection + RoPE + KV append 7B layer M={M} (packed heads)",
                  "kernel": "wsgemm_kernel (EPI_QKV)", "us": round(us, 2), "bytes": byt,
                  "achieved_gbs": round(byt / us / 1e3, 1), "peak_gbs": hbm,
                  "frac": round(byt / us / 1e3 / hbm, 4), "bound": "hbm",
                  "cublas_plus_rope_kv_append_us": round(us_two, 2),
                  "l2": "steady state over 6 weight sets (604 MB > L2)"})
            del kc, vc
        del ws, pws
    if not only or "prefill" in only:
        torch.manual_seed(1)
        q, k, v = (torch.randn(4, 32, 2048, 128, device=dev).to(torch.bfloat16) for _ in range(3))
        us = _time_us(lambda: flash_attention_v2(q, k, v, causal=True,
                                                 sm_scale=1 / math.sqrt(128)), 20)
        fl = 2 * 4 * 32 * 2048 * 2048 * 128
        emit({"op": "prefill attention [4,32,2048,128] causal bf16", "kernel": "flash_prefill_kernel",
              "us": round(us, 2), "flops": fl, "tflops": round(fl / us / 1e6, 1), "peak_tflops": tc,
              "frac": round(fl / us / 1e6 / tc, 4), "bound": "tensor",
              "flop_model": "2*B*H*S^2*D (benchmark_attention.py:104-116)",
              "l2": "inputs 201 MB > L2"})
    if not only or "decode" in only:
        torch.manual_seed(2)
        B, H, D = args.decode_batch, 32, 128
        L = torch.randint(128, 4097, (B,))
        Smax = 4097
        kc = torch.randn(B, H, Smax, D, device=dev, dtype=torch.bfloat16)
        vc = torch.randn(B, H, Smax, D, device=dev, dtype=torch.bfloat16)
        qkv = torch.randn(B, 1, 3 * H * D, device=dev).to(torch.bfloat16)
        cos, sin = precompute_freqs_cis(D, Smax, device=dev)
        cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
        pos = L.view(B, 1).to(dev)
        lens = (L + 1).to(torch.int32).to(dev)
        ws = ops.decode_attention_workspace(B, H, Smax, D, dev)
        outb = torch.empty(B, H, D, device=dev, dtype=torch.bfloat16)

        def step():
            qq = ops.rope_kv_append(qkv, pos, cos, sin, kc, vc, H, H)
            ops.decode_attention(qq.view(B, H, D), kc, vc, lens, None, outb, ws)

        us = _time_us(step, 20, flush)
        byt = int((L + 1).sum()) * H * D * 2 * 2 + 3 * B * H * D * 2 * 2
        emit({"op": f"decode step {B} ragged seqs L~U[128,4096] (rope+append+attention)",
              "kernel": "rope_kv_append_kernel + decode_split_kernel + decode_combine_kernel",
              "us": round(us, 2), "bytes": byt, "achieved_gbs": round(byt / us / 1e3, 1),
              "peak_gbs": hbm, "frac": round(byt / us / 1e3 / hbm, 4), "bound": "hbm",
              "l2": "flushed between launches"})
        us_a = _time_us(lambda: ops.decode_attention(qkv.view(B, 3, H, D)[:, 0], kc, vc, lens, None,
                                                     outb, ws), 20, flush)
        emit({"op": "decode attention only (same state)", "kernel": "decode_split+combine",
              "us": round(us_a, 2), "achieved_gbs": round(byt / us_a / 1e3, 1),
              "frac": round(byt / us_a / 1e3 / hbm, 4), "bound": "hbm"})
    return out


# ---------------------------------------------------------------------------
# long-context mixed run (--suite longctx)
# ---------------------------------------------------------------------------
LONG_SEQS, LONG_MIN, LONG_MAX, LONG_NEW, LONG_SEED = 64, 1024, 8192, 256, 4
KV_BYTES_PER_TOKEN_7B = 32 * 2 * 32 * 128 * 2   # 32 layers x (K, V) x 32 heads x 128 x bf16
WEIGHT_BYTES_7B = 13.215e9                      # all layers + lm_head, bf16


def long_prompts():
    """64 prompts of 1024..8192 tokens (uniform), ids uniform over the vocabulary."""
    g = torch.Generator().manual_seed(LONG_SEED)
    lens = torch.randint(LONG_MIN, LONG_MAX + 1, (LONG_SEQS,), generator=g).tolist()
    return [torch.randint(0, 32000, (n,), generator=g).tolist() for n in lens]


def lpt_partition(weights, world):
    """Longest-processing-time-first: heaviest sequence to the least-loaded rank."""
    loads = [0] * world
    parts = [[] for _ in range(world)]
    for i in sorted(range(len(weights)), key=lambda i: (-weights[i], i)):
        r = min(range(world), key=lambda r: (loads[r], r))
        parts[r].append(i)
        loads[r] += weights[i]
    return [sorted(p) for p in parts], loads


def run_longctx(args, world, rank, local):
    line = longctx_measure(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if line.get("device_status"):
        raise SystemExit(3)


def longctx_measure(args, world, rank, local):
    """The long-context mixed run on this rank's LPT share; every rank takes
    the same collective steps and returns the same line."""
    from llama_pure_compute_b200 import _lib
    from llama_pure_compute_b200.generate import BatchedGreedyDecoder
    from llama_pure_compute_b200.model import LlamaForCausalLM
    from llama_pure_compute_b200.ragged_cache import RaggedKVCache

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _lib.load()
    prompts = long_prompts()
    lens = [len(p) for p in prompts]
    parts, loads = lpt_partition([n + LONG_NEW for n in lens], world)
    mine = parts[rank]
    cfg = model_config(args.layers, LONG_MAX + LONG_NEW)
    model = LlamaForCausalLM.random_init(cfg, device=dev, dtype=torch.bfloat16, seed=SEED)
    cache = RaggedKVCache(num_layers=cfg.num_layers, capacities=[lens[i] + LONG_NEW for i in mine],
                          n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                          dtype=torch.bfloat16, device=dev)
    free, _ = torch.cuda.mem_get_info(dev)
    # packed weight copies for the decode-sized kernels, per layer: q/k/v
    # 100.7 MB, gate/up 180.4 MB, o_proj 33.6 MB + down_proj 90.2 MB; each is
    # kept only when this rank's step uses it and 2 GB stay free
    from llama_pure_compute_b200 import model as model_mod
    n, L, spare = len(mine), cfg.num_layers, free - 2e9
    use = {}
    for name, limit, nbytes in (("qkv", model_mod.FUSED_QKV_MAX_TOKENS, 100.7e6),
                                ("swiglu", model_mod.PACKED_SWIGLU_MAX_TOKENS, 180.4e6),
                                ("residual", model_mod.PACKED_RESIDUAL_MAX_TOKENS, 123.8e6)):
        use[name] = n <= limit and spare > L * nbytes
        if use[name]:
            spare -= L * nbytes
    mm = model.model
    mm.fused_qkv_max_tokens = model_mod.FUSED_QKV_MAX_TOKENS if use["qkv"] else 0
    mm.packed_swiglu_max_tokens = model_mod.PACKED_SWIGLU_MAX_TOKENS if use["swiglu"] else 0
    mm.packed_residual_max_tokens = model_mod.PACKED_RESIDUAL_MAX_TOKENS if use["residual"] else 0
    packed = use
    dec = BatchedGreedyDecoder(model, cache, len(mine), use_cuda_graph=True, prefill_chunk=1)

    barrier(world)
    clocks = ClockSampler(smi_index(local))
    clocks.start()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record()
    dec.prefill([prompts[i] for i in mine])
    p1.record()
    barrier(world)
    prefill_ms = max_over_ranks(p0.elapsed_time(p1), world)
    dec.capture()  # one untimed warm-up step inside, state restored
    barrier(world)
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(LONG_NEW):
        dec.graph.replay()
    d1.record()
    barrier(world)
    decode_ms = max_over_ranks(d0.elapsed_time(d1), world)
    clk = clocks.stop()
    status = int(max_over_ranks(float(_lib.device_status()), world))
    kv_gb = round(cache.memory_footprint_bytes() / 1e9, 2)
    dec.release()
    del dec, cache, model
    torch.cuda.empty_cache()

    sum_p = sum(lens)
    prefill_flops = 2 * 6.476e9 * sum_p + 2 * 32 * 128 * 32 * sum(n * n for n in lens)
    decode_tokens = LONG_SEQS * LONG_NEW
    # bytes per decode step, summed over ranks: each rank streams the weights
    # once plus its sequences' K/V (mean context P + 128 over the 256 steps)
    kv_bytes = sum(n + LONG_NEW // 2 for n in lens) * KV_BYTES_PER_TOKEN_7B
    step_bytes = world * WEIGHT_BYTES_7B + kv_bytes
    pk = _peaks()
    hbm = pk.get("hbm_gbs_sustained", pk.get("hbm_gbs", 6650.0))
    tc = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops", 1590.0))
    step_ms = decode_ms / LONG_NEW
    achieved = step_bytes / world / (step_ms / 1e3) / 1e9
    line = {
        "metric": "long-context mixed run: prefill tok/s and decode tok/s (7B shape)",
        "suite": "longctx", "value": round(decode_tokens / (decode_ms / 1e3), 1), "unit": "tok/s",
        "n_gpus": world, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform random prompt ids)",
        "config": {"workload": "64 prompts of 1024..8192 tokens (uniform, seed 4), prefill then "
                               "256 greedy decode steps, ragged KV cache",
                   "sum_prompt_tokens": sum_p, "prompt_len_min": min(lens),
                   "prompt_len_max": max(lens), "partition": "LPT on prompt+256",
                   "rank_loads": loads, "kv_cache_gb_rank0": kv_gb,
                   "packed_copies": packed},
        "prefill": {"tokens": sum_p, "ms": round(prefill_ms, 1),
                    "tok_s": round(sum_p / (prefill_ms / 1e3), 1),
                    "tflops": round(prefill_flops / (prefill_ms / 1e3) / 1e12 / world, 1),
                    "frac_tc_per_gpu": round(prefill_flops / (prefill_ms / 1e3) / 1e12 / world / tc, 4),
                    "flop_model": "2*6.476e9*sum(P) + 2*H*D*L*sum(P^2)"},
        "decode": {"steps": LONG_NEW, "ms": round(decode_ms, 1), "ms_per_step": round(step_ms, 3),
                   "tok_s": round(decode_tokens / (decode_ms / 1e3), 1),
                   "bytes_per_step_all_ranks": int(step_bytes),
                   "achieved_gbs_per_gpu": round(achieved, 1), "peak_gbs": hbm,
                   "frac_hbm": round(achieved / hbm, 4)},
        "clocks": clk, "device_status": status,
    }
    return line


def main():
    args = parse()
    if args.suite == "ops":
        run_ops(args)
        return
    if args.suite == "kernels":
        torch.cuda.set_device(0)
        only = set(filter(None, args.only.split(","))) or None
        for e in measure_kernels(torch.device("cuda", 0), only):
            print(json.dumps(e), flush=True)
        return
    if args.suite == "longctx":
        world, rank, local = dist_setup()
        try:
            run_longctx(args, world, rank, local)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
        return
    world, rank, local = dist_setup() if torch.cuda.is_available() else (1, 0, 0)
    if args.impl == "reference":
        try:
            run_reference(args, world, rank)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
        return
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        sys.exit(1)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
