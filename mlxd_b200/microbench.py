"""Decode-GEMV microbenchmark (the qmv measurement of the decoder step).

Times the 4-bit decode GEMV of libmlxd_cuda at a model's projection shapes
with CUDA events inside the library (mlxd_cuda_linear_timed). Weights are
rotated over copies that together exceed the 126 MB L2, so every launch
streams its weights from HBM. Achieved GB/s = algorithmic bytes (packed
weights + bf16 scale/bias per group + x in + y out) / mean launch time.

    python -m mlxd_b200.microbench [--shape gate_up] [--iters N] [--copies C]
"""
import argparse
import json

from . import cuda

QWEN3_8B = dict(hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                vocab=151936)


def shapes_of(kw):
    H, D = kw["hidden"], kw["head_dim"]
    q, kv = kw["n_heads"] * D, kw["n_kv_heads"] * D
    return {"qkv": (q + 2 * kv, H), "o_proj": (H, q), "gate_up": (2 * kw["inter"], H),
            "down": (H, kw["inter"]), "lm_head": (kw["vocab"], H)}


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
    for l in lins:
        l.close()
    gbs = wbytes / (ms * 1e-3) / 1e9
    return {"rows": rows, "cols": cols, "us": round(ms * 1e3, 2), "bytes": wbytes,
            "gbs": round(gbs, 1), "copies": copies, "iters": iters}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="all")
    ap.add_argument("--iters", type=int, default=None)
    ap.add_argument("--copies", type=int, default=None)
    args = ap.parse_args()
    cuda.init(0)
    shp = shapes_of(QWEN3_8B)
    names = list(shp) if args.shape == "all" else [args.shape]
    out = {n: measure(*shp[n], iters=args.iters, copies=args.copies) for n in names}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
