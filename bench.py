"""Decode benchmark of the mlxd decoder step on B200.

Workload (N=1 default): Qwen3-8B architecture, MLX affine 4-bit (group 64,
bf16 scales/biases) on seeded synthetic N(0, 0.02) weights, a 2048-token
uniform-random prompt, then greedy decode at batch 1. A "step" is one decode
token (one forward + token choice). W warm-up steps run untimed, then exactly K
steps are timed on the device with CUDA events (per-step events recorded on
the decode stream by the library). With --gpus N > 1 (torchrun) the model is
tensor parallel over N GPUs (NCCL allreduce after o_proj and down_proj);
the metric is the whole job's token rate (strong scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

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

WORKLOADS = {
    # name: (config kwargs, prompt, decode tokens in the reference workload)
    "qwen3-8b-4bit": (dict(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128,
                           inter=12288, vocab=151936, tie=False), 2048, 512),
    "qwen3-0.6b-4bit": (dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128,
                             inter=3072, vocab=151936, tie=True), 512, 256),
}
MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0


def metric_name(workload):
    if workload == "qwen3-8b-4bit":
        return "decode tokens/s at batch 1 (Qwen3-8B 4-bit)"
    return "decode tokens/s at batch 1 (%s)" % workload


def env_rank():
    r = int(os.environ.get("RANK", "0"))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", str(r)))
    return r, w, lr


def hbm_peak():
    try:
        d = json.load(open(MEASURED_PEAKS))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def bytes_per_token(kw, ctx, group=64):
    """Algorithmic HBM bytes of one decode token: every quantized weight once
    (4 bits + bf16 scale and bias per group), the KV cache read, one embed row."""
    H, L, D = kw["hidden"], kw["layers"], kw["head_dim"]
    q, kv = kw["n_heads"] * D, kw["n_kv_heads"] * D
    per_layer = (q + 2 * kv) * H + H * q + 2 * kw["inter"] * H + H * kw["inter"]
    params = L * per_layer + kw["vocab"] * H
    wbytes = params * (0.5 + 4.0 / group)
    kvbytes = L * 2 * kv * 2 * ctx
    return wbytes + kvbytes + H * (0.5 + 4.0 / group), wbytes


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
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
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
    """Element-wise max of per-rank device times (the job is as slow as its
    slowest rank)."""
    import torch
    v = torch.tensor([float(x) for x in values], dtype=torch.float64)
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return [float(x) for x in v]


def gemv_roofline(kw, peak):
    """Live qGEMV microbench at the workload's projection shapes (weights
    rotated over copies larger than L2, CUDA events in the library)."""
    from mlxd_b200 import microbench
    out = {}
    for name, (rows, cols) in microbench.shapes_of(kw).items():
        if name == "lm_head":
            continue
        r = microbench.measure(rows, cols)
        r["frac"] = round(r["gbs"] / peak, 3)
        out[name] = r
    return out


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


def oracle_sample(kw, host_tensors, prompt_len, vocab, budget_s, threads=0):
    """Time the CPU oracle's decode on the same weights (bounded sample)."""
    from oracle import pyoracle as po
    from mlxd_b200 import cuda
    from tests.helpers import orc_config
    if threads:
        po.lib().orc_set_threads(threads)
    cfg = cuda.synth_config(**kw, max_pos=prompt_len + 64)
    orc = po.Oracle(orc_config(cfg), host_tensors)
    prompt = cuda.synth_prompt(prompt_len, vocab, seed=0)
    kv = orc.new_kv(prompt_len + 64)
    t0 = time.time()
    orc.forward(kv, prompt, want_logits=False)
    pre_s = time.time() - t0
    tok = int(prompt[-1])
    n, t_dec = 0, 0.0
    while t_dec < budget_s and n < 64:
        t1 = time.time()
        lg = orc.forward(kv, [tok])
        t_dec += time.time() - t1
        tok = int(np.argmax(lg))
        n += 1
    return {"value": round(n / t_dec, 4), "unit": "tokens/s", "cores": po.lib().orc_get_threads(),
            "kind": "port",
            "sample": "CPU oracle (C restatement, pthreads): %d-token prompt prefill (%.1f s, "
                      "untimed), then %d greedy decode tokens timed (%.1f s), same seeded "
                      "4-bit weights" % (prompt_len, pre_s, n, t_dec)}


def host_weights_from_gpu(cuda, cfg):
    dev = cuda.synth_device_tensors(cfg, seed=0)
    host = cuda.device_tensors_to_host(dev)
    for v in dev.values():
        v[0].free()
    return host


def run_reference(args, rank, world, lr):
    """The reference arm: tlkahn/mlxd itself cannot run here (mlx-c / Metal
    only), so the path's CPU implementation is the oracle port, timed on the
    host cores on the same workload (bounded sample)."""
    if rank != 0:
        return
    from mlxd_b200 import cuda
    kw, P, _ = WORKLOADS[args.workload]
    cfg = cuda.synth_config(**kw, max_pos=P + args.warmup + args.steps + 8)
    try:
        cuda.init(lr)
        host = host_weights_from_gpu(cuda, cfg)
    except Exception:
        host = cuda.synth_host_tensors(cfg, seed=0)
    cb = oracle_sample(kw, host, args.cpu_prompt, kw["vocab"], args.cpu_budget)
    line = {"impl": "reference", "metric": metric_name(args.workload), "value": cb["value"],
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "u4 weights / bf16 activations (f32 accumulate)",
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
    ap.add_argument("--cpu-prompt", type=int, default=8)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--roofline", type=int, default=1)
    ap.add_argument("--sampled", type=int, default=1,
                    help="also time sampled decoding (one GPU; temperature 0.7, top-k 50, top-p 0.9, "
                         "repetition penalty 1.1 over 256 tokens)")
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
    kw, P, _ = WORKLOADS[args.workload]
    if args.prompt:
        P = args.prompt
    K, W = args.steps, args.warmup
    total = W + K
    SAMPLED_STEPS, SAMPLED_WARMUP = 256, 16
    room = max(total, SAMPLED_STEPS + SAMPLED_WARMUP) + 8   # positions past the prompt
    cfg = cuda.synth_config(**kw, max_pos=P + room, tp_rank=rank, tp_size=world)
    t0 = time.time()
    dev = cuda.synth_device_tensors(cfg, seed=0)
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
    prompt = cuda.synth_prompt(P, cfg.vocab, seed=0)
    kv = model.new_kv(P + room)
    # untimed warm-up of the whole path (graph capture, allocator)
    model.generate(prompt[:64], 4, kv=kv)
    if dist:
        dist.barrier()
    clocks = ClockSampler(lr)
    clocks.start()
    toks, _, tm = model.generate(prompt, total, kv=kv)
    clk = clocks.stop()
    if len(toks) != total:
        raise SystemExit("decode stopped early (%d of %d tokens)" % (len(toks), total))
    ends = tm["step_end_ms"]
    t_timed = float(ends[total - 1] - ends[W - 1])          # exactly K steps
    wall_ms = float(tm["decode_wall_ms"])
    prefill_ms = float(tm["prefill_ms"])
    if dist:
        t_timed, wall_ms, prefill_ms = max_over_ranks(dist, [t_timed, wall_ms, prefill_ms])
    value = K / (t_timed / 1e3)
    e2e_value = total / (wall_ms / 1e3)
    peak, peak_src = hbm_peak()
    mean_ctx = P + W + K / 2.0
    bpt, wbytes = bytes_per_token(kw, mean_ctx)
    step_gbs = bpt / world / (t_timed / K / 1e3) / 1e9
    line = {
        "metric": metric_name(args.workload),
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(t_timed / K, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "u4 weights / bf16 activations (f32 accumulate)",
        "data": "synthetic (seeded N(0,0.02) -> bf16 -> MLX affine 4-bit g64, uniform prompt ids)",
        "config": {"workload": args.workload, "prompt": P, "decode_tokens": total, "batch": 1,
                   "parallelism": "tp%d" % world, "group": 64,
                   "l2": "weights %.2f GB per GPU > 126 MB L2 (no flush needed)" % (wbytes / world / 1e9),
                   "prefill_tokens_per_s": round((P - 1) / (prefill_ms / 1e3), 1),
                   "model_load_s": round(load_s, 1)},
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4,
                "how": "host wall clock of the mlxd_cuda_generate decode loop (C ABI, host "
                       "prompt in, one 4-byte token read back per step); prompt H2D and "
                       "prefill are reported as prefill_tokens_per_s"},
        "step_roofline": {"bytes_per_token": round(bpt / world), "achieved_gbs": round(step_gbs, 1),
                          "peak_gbs": peak, "peak_source": peak_src,
                          "frac": round(step_gbs / peak, 4), "mean_context": mean_ctx},
        "gpu_launches": K * (1 + 5 * kw["layers"] + 2 + (2 * kw["layers"] if world > 1 else 0)),
        "clocks": clk,
    }
    if args.sampled and world == 1:
        # sampled decoding (the Mistral-style workload's settings) on the same
        # model and prompt: one captured step (forward, sampler, append) per
        # token, device time between the first and last timed step
        sp = cuda.sampling(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1,
                           repetition_context=256, seed=1)
        ns, ws = SAMPLED_STEPS, SAMPLED_WARMUP
        model.generate(prompt[:64], 4, sp=sp, kv=kv)
        stoks, _, stm = model.generate(prompt, ws + ns, sp=sp, kv=kv)
        if len(stoks) == ws + ns:
            se = stm["step_end_ms"]
            line["config"]["sampled_decode"] = {
                "tokens_per_s": round(ns / (float(se[ws + ns - 1] - se[ws - 1]) / 1e3), 2),
                "steps": ns, "warmup": ws,
                "settings": "temperature 0.7, top_k 50, top_p 0.9, repetition_penalty 1.1 (last 256)"}
    if args.roofline and rank == 0:
        g = gemv_roofline(kw, peak)
        dom = g["gate_up"]
        tr = load_traffic().get("gate_up")
        line["roofline"] = {"kernel": "qgemv (decode 4-bit GEMV), gate_up shape %dx%d" % (
            dom["rows"], dom["cols"]), "bound": "hbm", "achieved": dom["gbs"], "peak": peak,
            "unit": "GB/s", "frac": round(dom["gbs"] / peak, 4),
            "traffic": round(tr["bytes_per_launch"]) if tr else None,
            "traffic_note": ("DRAM bytes read+written per launch, one ncu capture of this shape (%s); "
                             "algorithmic bytes %d" % (tr["source"], dom["bytes"])) if tr else None,
            "peak_source": peak_src, "shapes": g}
    if args.cpu_baseline and rank == 0 and world == 1:
        try:
            host = host_weights_from_gpu(cuda, cuda.synth_config(**kw, max_pos=P + room))
            line["cpu_baseline"] = oracle_sample(kw, host, args.cpu_prompt, kw["vocab"],
                                                 args.cpu_budget)
            del host
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
