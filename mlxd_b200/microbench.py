"""Decode-GEMV microbenchmark (the qmv measurement of the decoder step).

Times the 4-bit decode GEMV of libmlxd_cuda at a model's projection shapes
with CUDA events inside the library: launched alone (mlxd_cuda_linear_timed)
and chained to the previous launch by programmatic dependent launch as in
the decode step's graph (mlxd_cuda_linear_timed_chained). Weights are
rotated over copies that together exceed the 126 MB L2, so every launch
streams its weights from HBM. Achieved GB/s = algorithmic bytes (packed
weights + bf16 scale/bias per group + x in + y out) / mean launch time.

    python -m mlxd_b200.microbench [--shape gate_up] [--iters N] [--copies C]
    python -m mlxd_b200.microbench --prefill-gemm   # tcgen05 GEMM, 24576 x 4096, 512 tokens
    python -m mlxd_b200.microbench --attention      # decode attention, 32/8 heads, context 2048
    python -m mlxd_b200.microbench --prefill-layer  # chunked 2048-token prefill of one Qwen3-8B layer
    python -m mlxd_b200.microbench --sampler        # sampler, V 151936, T 0.7 k 50 p 0.9 rep 1.1
"""
import argparse
import json

from . import cuda

QWEN3_8B = dict(hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                vocab=151936)


def shapes_of(kw, tp=1):
    """Decode projection shapes (rows, cols) of one rank at tensor-parallel
    degree tp: q/k/v, gate/up and lm_head split by rows, o and down by
    columns."""
    H, D = kw["hidden"], kw["head_dim"]
    q, kv = kw["n_heads"] * D // tp, kw["n_kv_heads"] * D // tp
    return {"qkv": (q + 2 * kv, H), "o_proj": (H, q), "gate_up": (2 * kw["inter"] // tp, H),
            "down": (H, kw["inter"] // tp), "lm_head": (kw["vocab"] // tp, H)}


def gemv_bytes(rows, cols, group=64):
    return rows * cols // 2 + rows * (cols // group) * 4 + cols * 2 + rows * 2


def measure(rows, cols, iters=None, copies=None, group=64, min_bytes=400e6):
    wbytes = gemv_bytes(rows, cols, group)
    if copies is None:
        copies = max(2, int(min_bytes // wbytes) + 1)
    if iters is None:
        iters = max(3, 200 // copies)
    x = cuda.DeviceBuffer(cols * 2)
    cuda.check(cuda.lib().mlxd_cuda_synth_bf16(x.ptr, cols, 99, 1.0, 0.0, None), "synth")
    y = cuda.DeviceBuffer(rows * 2)
    lins = []
    for c in range(copies):
        w = cuda.DeviceBuffer(rows * cols // 2)
        s = cuda.DeviceBuffer(rows * cols // group * 2)
        b = cuda.DeviceBuffer(rows * cols // group * 2)
        cuda.check(cuda.lib().mlxd_cuda_synth_quantized(w.ptr, s.ptr, b.ptr, rows, cols, group,
                                                        1000 + c, 0.02, None), "synth")
        lins.append(cuda.Linear(w, s, b, group, rows=rows, cols=cols))
        w.free(), s.free(), b.free()
    ms = cuda.linear_timed(lins, iters, x, y)
    ms_c = cuda.linear_timed(lins, iters, x, y, chained=True)
    for l in lins:
        l.close()
    gbs = wbytes / (ms * 1e-3) / 1e9
    return {"rows": rows, "cols": cols, "us": round(ms * 1e3, 2), "bytes": wbytes,
            "gbs": round(gbs, 1), "copies": copies, "iters": iters,
            "chained_us": round(ms_c * 1e3, 2), "chained_gbs": round(wbytes / (ms_c * 1e-3) / 1e9, 1)}


def prefill_gemm(rows=24576, cols=4096, S=512, reps=3):
    """The prefill GEMM (mlxd_cuda_linear with S tokens) on one synthetic
    group-64 matrix, `reps` launches; for ncu captures of the tcgen05 kernel."""
    import numpy as np
    w = cuda.DeviceBuffer(rows * cols // 2)
    s = cuda.DeviceBuffer(rows * cols // 64 * 2)
    b = cuda.DeviceBuffer(rows * cols // 64 * 2)
    cuda.check(cuda.lib().mlxd_cuda_synth_quantized(w.ptr, s.ptr, b.ptr, rows, cols, 64, 5, 0.02, None),
               "synth")
    lin = cuda.Linear(w, s, b, 64, rows=rows, cols=cols)
    x = np.random.default_rng(0).standard_normal((S, cols)).astype(np.float32)
    xb = (x.view(np.uint32) >> 16).astype(np.uint16)
    for _ in range(reps):
        y = lin(xb)
    lin.close()
    return {"prefill_gemm": {"rows": rows, "cols": cols, "tokens": S, "launches": reps,
                             "out_shape": list(y.shape)}}


def decode_attention(context=2048, steps=6):
    """Decode steps of a 2-layer model with the Qwen3-8B attention shape (32/8
    heads, head_dim 128) after a `context`-token prefill, through
    mlxd_cuda_forward; for ncu captures of the decode attention kernel."""
    import numpy as np
    cfg = cuda.synth_config(hidden=1024, layers=2, n_heads=32, n_kv_heads=8, head_dim=128, inter=1024,
                            vocab=4096, max_pos=context + steps + 64)
    m = cuda.Model(cfg, cuda.synth_host_tensors(cfg, seed=1))
    kv = m.new_kv(context + steps + 64)
    ids = np.random.default_rng(0).integers(0, cfg.vocab, context).tolist()
    m.forward(kv, ids, want_logits=False)
    t = 5
    for _ in range(steps):
        t = int(np.argmax(m.forward(kv, [t])))
    m.close()
    return {"decode_attention": {"context": context, "steps": steps, "last_token": t}}


def prefill_layer(prompt=2048, chunk=512):
    """A chunked prefill of `prompt` tokens through one Qwen3-8B-shaped decoder
    layer (vocab 1024, so the projections, attention and norms dominate), for
    launch lists of the prefill's kernels."""
    cfg = cuda.synth_config(hidden=4096, layers=1, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                            vocab=1024, max_pos=prompt + 64)
    dev = cuda.synth_device_tensors(cfg, seed=0)
    m = cuda.Model(cfg, dev, on_device=True)
    for v in dev.values():
        v[0].free()
    kv = m.new_kv(prompt + 64)
    ids = cuda.synth_prompt(prompt, cfg.vocab, 0).tolist()
    for a in range(0, prompt, chunk):
        m.forward(kv, ids[a:a + chunk], want_logits=False)
    cuda.synchronize()
    m.close()
    return {"prefill_layer": {"prompt": prompt, "chunk": chunk}}


SAMPLER_DEFAULT = dict(temperature=0.7, top_k=50, top_p=0.9, seed=7, repetition_penalty=1.1,
                      repetition_context=256)


def sampler(V=151936, reps=6, timed=50, settings=None):
    """The sampler (mlxd_cuda_sample) on one bf16 logits row of V entries with
    the sampled-decode settings of the Mistral-style workload: temperature 0.7,
    top-k 50, top-p 0.9, repetition penalty 1.1 over the last 256 context
    tokens (or `settings`); `reps` draws reported, then `timed` back-to-back
    draws on the default stream between two CUDA events (the mean device time
    per draw)."""
    import ctypes as C
    import numpy as np
    import torch
    rng = np.random.default_rng(0)
    logits = (rng.standard_normal(V).astype(np.float32) * 3.0)
    lb = (logits.view(np.uint32) >> 16).astype(np.uint16)
    ctx = rng.integers(0, V, 256).astype(np.int32)
    settings = dict(SAMPLER_DEFAULT if settings is None else settings)
    sp = cuda.sampling(**settings)
    dl = cuda.DeviceBuffer.from_array(lb)
    dc = cuda.DeviceBuffer.from_array(ctx)
    tok = cuda.DeviceBuffer(4)
    L = cuda.lib()

    def draw(step):
        cuda.check(L.mlxd_cuda_sample(dl.ptr, cuda.BF16, V, C.byref(sp), dc.ptr, len(ctx), step, tok.ptr,
                                      None, None, None), "sample")
    toks = []
    for r in range(reps):
        draw(r)
        toks.append(int(tok.to_array(np.int32, (1,))[0]))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cuda.check(L.mlxd_cuda_synchronize(None), "sync")
    e0.record(torch.cuda.default_stream())
    for r in range(timed):
        draw(reps + r)
    e1.record(torch.cuda.default_stream())
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / timed
    return {"sampler": {"V": V, "settings": settings, "draws": reps, "tokens": toks, "us_per_draw": round(us, 2),
                        "timed_draws": timed}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="all")
    ap.add_argument("--iters", type=int, default=None)
    ap.add_argument("--copies", type=int, default=None)
    ap.add_argument("--prefill-gemm", action="store_true", help="run the tcgen05 prefill GEMM workload")
    ap.add_argument("--attention", action="store_true", help="run the decode attention workload")
    ap.add_argument("--prefill-layer", action="store_true",
                    help="chunked 2048-token prefill through one Qwen3-8B-shaped layer")
    ap.add_argument("--sampler", action="store_true", help="run the sampler on a 151936-entry row")
    ap.add_argument("--sampler-settings", default=None,
                    help="JSON sampling settings for --sampler (default: the sampled-decode settings)")
    args = ap.parse_args()
    cuda.init(0)
    if args.prefill_gemm:
        print(json.dumps(prefill_gemm()))
        return
    if args.attention:
        print(json.dumps(decode_attention()))
        return
    if args.prefill_layer:
        print(json.dumps(prefill_layer()))
        return
    if args.sampler:
        print(json.dumps(sampler(settings=json.loads(args.sampler_settings) if args.sampler_settings else None)))
        return
    shp = shapes_of(QWEN3_8B)
    names = list(shp) if args.shape == "all" else [args.shape]
    out = {n: measure(*shp[n], iters=args.iters, copies=args.copies) for n in names}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
