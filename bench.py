"""Decode benchmark of the mlxd decoder step on B200.

Workloads (synthetic seeded N(0, 0.02) weights, MLX affine 4-bit group 64 with
bf16 scales/biases, uniform-random prompt ids):

  qwen3-8b-4bit     (default) Qwen3-8B, 2048-token prompt, greedy decode
  qwen3-0.6b-4bit   Qwen3-0.6B, 512-token prompt, greedy decode
  qwen3-tiny-4bit   2 layers, hidden 64, 16-token prompt, greedy decode
  mistral-7b-4bit   Mistral-7B, sliding window 4096 (ring of 4607 slots),
                    8192-token prompt in 512-token chunks, sampled decode
                    (temperature 0.7, top-k 50, top-p 0.9, repetition 1.1)
  llama3-70b-4bit   Llama-3-70B (llama3-scaled RoPE), 4096-token prompt,
                    greedy decode; tensor parallel with --gpus N

A "step" is one decode token (one forward + token choice). W warm-up steps run
untimed, then exactly K steps are timed on the device with CUDA events
(per-step events recorded on the decode stream by the library). With --gpus
N > 1 (torchrun) the model is tensor parallel over N GPUs; the row-parallel
sums, the greedy argmax and the sampler's logits travel over NVLink inside the
captured step. `value` is the whole job's token rate (strong scaling).

`e2e` is the same metric through the public generate call with host buffers:
prompt ids uploaded from host memory, chunked prefill, then the decode loop
reading back one 4-byte token per step, timed by the host clock around the
call. `prefill_roofline` is the prefill's FLOPs over the measured sustained
bf16 tensor peak. `roofline` is the dominant kernel (the gate|up decode GEMV
shape) timed with CUDA events over back-to-back launches chained by
programmatic dependent launch, the decode graph's launch mode; every
projection shape's rate launched alone and chained is in `roofline.shapes`.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                  [--impl reference]

Prints one JSON line (rank 0).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

QWEN3, LLAMA, MISTRAL = 1, 2, 3
SAMPLED = dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1, repetition_context=256,
               seed=1)

WORKLOADS = {
    # name: config kwargs, prompt length, decode tokens in the workload,
    # sampling settings (None: greedy), prefill chunk, KV ring slots
    "qwen3-8b-4bit": dict(kw=dict(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128,
                                  inter=12288, vocab=151936, tie=False),
                          prompt=2048, decode=512, sampling=None),
    "qwen3-0.6b-4bit": dict(kw=dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128,
                                    inter=3072, vocab=151936, tie=True),
                            prompt=512, decode=256, sampling=None),
    "qwen3-tiny-4bit": dict(kw=dict(hidden=64, layers=2, n_heads=4, n_kv_heads=2, head_dim=16,
                                    inter=128, vocab=256, tie=True),
                            prompt=16, decode=32, sampling=None),
    "mistral-7b-4bit": dict(kw=dict(hidden=4096, layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                                    inter=14336, vocab=32768, tie=False, family=MISTRAL, window=4096),
                            prompt=8192, decode=1024, sampling=SAMPLED, chunk=512),
    "llama3-70b-4bit": dict(kw=dict(hidden=8192, layers=80, n_heads=64, n_kv_heads=8, head_dim=128,
                                    inter=28672, vocab=128256, tie=False, family=LLAMA, theta=500000.0,
                                    llama3=(8.0, 1.0, 4.0, 8192)),
                            prompt=4096, decode=512, sampling=None),
}
MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops_sustained": 1400.0}


def metric_name(workload):
    names = {"qwen3-8b-4bit": "Qwen3-8B 4-bit", "qwen3-0.6b-4bit": "Qwen3-0.6B 4-bit",
             "qwen3-tiny-4bit": "tiny Qwen3 4-bit", "mistral-7b-4bit": "Mistral-7B 4-bit, window 4096, sampled",
             "llama3-70b-4bit": "Llama-3-70B 4-bit"}
    return "decode tokens/s at batch 1 (%s)" % names[workload]


def env_rank():
    r = int(os.environ.get("RANK", "0"))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", str(r)))
    return r, w, lr


def peaks():
    try:
        d = json.load(open(MEASURED_PEAKS))
        return float(d["hbm_gbs"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return FALLBACK["hbm_gbs"], FALLBACK["bf16_tflops_sustained"], "fallback"


def proj_params(kw):
    """Quantized projection parameters of one decoder layer."""
    H, D = kw["hidden"], kw["head_dim"]
    q, kv = kw["n_heads"] * D, kw["n_kv_heads"] * D
    return (q + 2 * kv) * H + H * q + 3 * kw["inter"] * H


def bytes_per_token(kw, ctx, group=64):
    """Algorithmic HBM bytes of one decode token: every quantized weight once
    (4 bits + bf16 scale and bias per group), the KV cache read over the
    attended context (the window, if any), one embed row."""
    H, L, D = kw["hidden"], kw["layers"], kw["head_dim"]
    kv = kw["n_kv_heads"] * D
    if kw.get("window"):
        ctx = min(ctx, kw["window"])
    params = L * proj_params(kw) + kw["vocab"] * H
    wbytes = params * (0.5 + 4.0 / group)
    kvbytes = L * 2 * kv * 2 * ctx
    return wbytes + kvbytes + H * (0.5 + 4.0 / group), wbytes


def prefill_flops(kw, n):
    """FLOPs of a prefill of n tokens without logits: 2 per weight per token
    for the projections, and 4 * head_dim per (query head, key) pair for the
    causal (or windowed) attention."""
    L, D, hq = kw["layers"], kw["head_dim"], kw["n_heads"]
    w = kw.get("window") or 0
    keys = sum(min(t, w) if w else t for t in range(1, n + 1))
    return 2.0 * n * L * proj_params(kw) + 4.0 * D * hq * L * keys


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=5)
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


def dist_setup(world):
    if world <= 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return dist


def max_over_ranks(dist, values):
    """Element-wise max of per-rank times (the job is as slow as its slowest
    rank)."""
    import torch
    v = torch.tensor([float(x) for x in values], dtype=torch.float64)
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return [float(x) for x in v]


def gemv_roofline(kw, peak, tp):
    """Live decode-GEMV microbench at this rank's projection shapes (weights
    rotated over copies larger than L2, CUDA events in the library)."""
    from mlxd_b200 import microbench
    out = {}
    for name, (rows, cols) in microbench.shapes_of(kw, tp).items():
        r = microbench.measure(rows, cols)
        r["frac"] = round(r["gbs"] / peak, 3)
        r["chained_frac"] = round(r["chained_gbs"] / peak, 3)
        out[name] = r
    return out


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


def model_config(cuda, wl, max_pos, rank=0, world=1):
    kw = dict(wl["kw"])
    return cuda.synth_config(**kw, max_pos=max_pos, tp_rank=rank, tp_size=world)


def kv_slots(wl, prompt, room):
    w = wl["kw"].get("window")
    return w + wl.get("chunk", 512) - 1 if w else prompt + room


def oracle_decode_sample(wl, prompt, budget_s, max_tokens, threads=0):
    """The CPU oracle's decode step on the workload's model (weights from the
    oracle's own copy of the seeded generator; no CUDA library in this
    process), at the workload's context: the cache is filled with seeded
    keys/values for the prompt's positions in place of a CPU prefill (the
    step's cost does not depend on the cached values), then decode tokens
    are timed until the budget or max_tokens."""
    from oracle import pyoracle as po
    from mlxd_b200 import cuda   # ctypes structs and tensor names only
    from tests.helpers import orc_config
    if threads:
        po.lib().orc_set_threads(threads)
    kw = wl["kw"]
    cfg = model_config(cuda, wl, prompt + max_tokens + 8)
    t0 = time.time()
    host = po.synth_host_tensors(cuda.synth_tensor_specs(cfg), cfg.qgroup, seed=0)
    orc = po.Oracle(orc_config(cfg), host)
    del host
    synth_s = time.time() - t0
    kv = orc.new_kv(prompt + max_tokens + 8)
    po.lib().orc_kv_fill_synth(kv.kv, prompt - 1, 7)
    tok = int(cuda.synth_prompt(prompt, cfg.vocab, seed=0)[-1])
    n, t_dec = 0, 0.0
    while t_dec < budget_s and n < max_tokens:
        t1 = time.time()
        lg = orc.forward(kv, [tok])
        t_dec += time.time() - t1
        tok = int(np.argmax(lg))
        n += 1
    ctx = prompt if not kw.get("window") else min(prompt, kw["window"])
    return {"value": round(n / t_dec, 4), "unit": "tokens/s", "cores": po.lib().orc_get_threads(),
            "kind": "port", "tokens": n, "seconds": round(t_dec, 2),
            "libmlxd_cuda_loaded": cuda._lib is not None,
            "sample": "CPU oracle (C restatement, pthreads) on the same seeded 4-bit weights (built "
                      "on the host in %.0f s): %d decode tokens timed at context %d (cache filled "
                      "with seeded keys/values for the %d prompt positions; attended context %d), "
                      "greedy" % (synth_s, n, prompt, prompt - 1, ctx)}


def run_reference(args, rank, world, lr):
    """The reference arm: tlkahn/mlxd itself cannot run here (mlx-c + Metal
    only), so the path's CPU implementation is the oracle port, timed on the
    host cores on the same workload (bounded sample). Rank 0 only."""
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    P = args.prompt or wl["prompt"]
    cb = oracle_decode_sample(wl, P, args.cpu_budget, max(1, min(args.steps, 64)))
    line = {"impl": "reference", "metric": metric_name(args.workload), "value": cb["value"],
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "u4 weights / bf16 activations",
            "data": "synthetic", "vs_baseline": None,
            "config": {"workload": args.workload, "prompt": P, "batch": 1,
                       "note": "reference engine needs mlx-c + Metal: unavailable on this box; "
                               "its CPU path is the oracle port"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=480)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen3-8b-4bit", choices=list(WORKLOADS))
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--cpu-baseline", type=int, default=1)
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--roofline", type=int, default=1)
    ap.add_argument("--sampled", type=int, default=1,
                    help="greedy workloads on one GPU: also time sampled decoding (temperature 0.7, "
                         "top-k 50, top-p 0.9, repetition penalty 1.1 over 256 tokens)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, lr = env_rank()
    if args.impl == "reference":
        run_reference(args, rank, world, lr)
        return
    from mlxd_b200 import cuda
    dist = dist_setup(world)
    cuda.init(lr)
    wl = WORKLOADS[args.workload]
    kw = wl["kw"]
    P = args.prompt or wl["prompt"]
    chunk = wl.get("chunk", 512)
    K, W = args.steps, args.warmup
    total = W + K
    SAMPLED_STEPS, SAMPLED_WARMUP = 256, 16
    room = max(total, SAMPLED_STEPS + SAMPLED_WARMUP) + 8   # positions past the prompt
    cfg = model_config(cuda, wl, P + room, rank, world)
    t0 = time.time()
    dev = cuda.synth_device_tensors(model_config(cuda, wl, P + room), seed=0)
    model = cuda.Model(cfg, dev, on_device=True)
    for v in dev.values():
        v[0].free()
    del dev
    load_s = time.time() - t0
    if world > 1:
        import torch
        uid = np.zeros(128, np.uint8)
        if rank == 0:
            cuda.check(cuda.lib().mlxd_cuda_nccl_unique_id(cuda.ptr(uid)), "nccl id")
        t = torch.from_numpy(uid.copy())
        dist.broadcast(t, 0)
        model.tp_init(t.numpy().tobytes())
    sp = cuda.sampling(**wl["sampling"]) if wl["sampling"] else None
    prompt = cuda.synth_prompt(P, cfg.vocab, seed=0)
    kv = model.new_kv(kv_slots(wl, P, room))
    # untimed warm-up of the whole path (graph capture, allocator)
    model.generate(prompt[:64], 4, sp=sp, kv=kv, chunk=chunk)
    if dist:
        dist.barrier()
    clocks = ClockSampler(lr)
    clocks.start()
    t_call = time.perf_counter()
    toks, _, tm = model.generate(prompt, total, sp=sp, kv=kv, chunk=chunk)
    call_ms = (time.perf_counter() - t_call) * 1e3
    clk = clocks.stop()
    if len(toks) != total:
        raise SystemExit("decode stopped early (%d of %d tokens)" % (len(toks), total))
    ends = tm["step_end_ms"]
    t_timed = float(ends[total - 1] - ends[W - 1])          # exactly K steps
    prefill_ms = float(tm["prefill_ms"])
    if dist:
        t_timed, call_ms, prefill_ms = max_over_ranks(dist, [t_timed, call_ms, prefill_ms])
    value = K / (t_timed / 1e3)
    hbm, tc_sust, peak_src = peaks()
    mean_ctx = P + W + K / 2.0
    bpt, wbytes = bytes_per_token(kw, mean_ctx)
    step_gbs = bpt / world / (t_timed / K / 1e3) / 1e9
    pf_flops = prefill_flops(kw, P - 1)
    pf_tflops = pf_flops / world / (prefill_ms / 1e3) / 1e12
    layers = kw["layers"]
    launches = 1 + 5 * layers + 2 + (2 * layers if world > 1 else 0)
    if sp is not None:
        launches += 6 + (1 if world > 1 else 0)
    line = {
        "metric": metric_name(args.workload),
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(t_timed / K, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "u4 weights / bf16 activations (exact integer group sums, f64 combination)",
        "data": "synthetic (seeded N(0,0.02) -> bf16 -> MLX affine 4-bit g64, uniform prompt ids)",
        "config": {"workload": args.workload, "prompt": P, "decode_tokens": total, "batch": 1,
                   "parallelism": "tp%d" % world, "group": 64, "prefill_chunk": chunk,
                   "decoding": "sampled: " + json.dumps(wl["sampling"]) if sp else "greedy",
                   "window": kw.get("window") or None, "kv_slots": kv_slots(wl, P, room),
                   "l2": "weights %.2f GB per GPU > 126 MB L2 (no flush needed)" % (wbytes / world / 1e9),
                   "model_load_s": round(load_s, 1)},
        "e2e": {"value": round(total / (call_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": round(4.0 * P / total, 2), "d2h_bytes_per_step": 4,
                "call_ms": round(call_ms, 1), "h2d_bytes_per_call": 4 * P,
                "includes": ["prompt ids H2D from host memory", "chunked prefill of %d tokens" % (P - 1),
                             "%d decode steps" % total, "4-byte token read back per step"],
                "how": "host clock around one mlxd_cuda_generate call (C ABI, host prompt in, host "
                       "tokens out); decode tokens / call time (max over ranks)"},
        "step_roofline": {"bytes_per_token": round(bpt / world), "achieved_gbs": round(step_gbs, 1),
                          "peak_gbs": hbm, "peak_source": peak_src,
                          "frac": round(step_gbs / hbm, 4), "mean_context": mean_ctx},
        "prefill_roofline": {"tokens_per_s": round((P - 1) / (prefill_ms / 1e3), 1),
                             "ms": round(prefill_ms, 2), "flops": pf_flops,
                             "achieved_tflops": round(pf_tflops, 1), "peak_tflops": tc_sust,
                             "peak": "bf16 dense, sustained (%s)" % peak_src,
                             "frac": round(pf_tflops / tc_sust, 4),
                             "note": "projections run on the integer tensor cores (tcgen05 kind::i8) "
                                     "in the exact arithmetic; FLOPs counted as bf16-equivalent"},
        "gpu_launches": K * launches,
        "clocks": clk,
    }
    if args.sampled and world == 1 and sp is None:
        # sampled decoding on the same model and prompt: one captured step
        # (forward, sampler, append) per token
        ssp = cuda.sampling(**SAMPLED)
        ns, ws = SAMPLED_STEPS, SAMPLED_WARMUP
        model.generate(prompt[:64], 4, sp=ssp, kv=kv, chunk=chunk)
        stoks, _, stm = model.generate(prompt, ws + ns, sp=ssp, kv=kv, chunk=chunk)
        if len(stoks) == ws + ns:
            se = stm["step_end_ms"]
            line["config"]["sampled_decode"] = {
                "tokens_per_s": round(ns / (float(se[ws + ns - 1] - se[ws - 1]) / 1e3), 2),
                "steps": ns, "warmup": ws, "settings": SAMPLED}
    if args.roofline and rank == 0:
        g = gemv_roofline(kw, hbm, world)
        dom = g["gate_up"]
        tr = load_traffic().get("gate_up") if world == 1 and args.workload == "qwen3-8b-4bit" else None
        line["roofline"] = {
            "kernel": "qgemv_i8 (decode 4-bit GEMV, plain prologue and store epilogue), gate_up shape %dx%d; "
                      "launches chained by programmatic dependent launch as in the decode graph (alone: "
                      "%.2f us, %.1f GB/s)" % (dom["rows"], dom["cols"], dom["us"], dom["gbs"]),
            "bound": "hbm", "achieved": dom["chained_gbs"], "peak": hbm,
            "unit": "GB/s", "frac": round(dom["chained_gbs"] / hbm, 4),
            "us_per_launch": dom["chained_us"], "alone_frac": round(dom["gbs"] / hbm, 4),
            "traffic": round(tr["bytes_per_launch"]) if tr else None,
            "traffic_note": ("DRAM bytes read+written per launch, one ncu capture of this shape (%s); "
                             "algorithmic bytes %d" % (tr["source"], dom["bytes"])) if tr else None,
            "peak_source": peak_src, "shapes": g}
    if args.cpu_baseline and rank == 0 and world == 1:
        try:
            line["cpu_baseline"] = oracle_decode_sample(wl, P, args.cpu_budget, 64)
        except Exception as e:  # reported, never silently dropped
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
