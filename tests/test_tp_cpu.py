"""Tensor parallel on the CPU: the library's shard plan (mlxd_cuda_tp_plan,
the partition mlxd_cuda_model_create applies) partitions every projection, and
two gloo ranks that each compute their shard of a quantized layer (numpy
dequantization, f32) and combine it the way the decode step does (all-reduce
of row-parallel partials, gather of column-parallel outputs) reproduce the
unsharded layer. No GPU is used."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from mlxd_b200 import cuda

QWEN3_8B = dict(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                vocab=151936, tie=False)
LLAMA3_70B = dict(hidden=8192, layers=80, n_heads=64, n_kv_heads=8, head_dim=128, inter=28672,
                  vocab=128256, tie=False)


def full_shapes(cfg):
    D, H = cfg.head_dim, cfg.hidden
    return {"q": (cfg.n_heads * D, H), "k": (cfg.n_kv_heads * D, H), "v": (cfg.n_kv_heads * D, H),
            "o": (H, cfg.n_heads * D), "gate": (cfg.inter, H), "up": (cfg.inter, H),
            "down": (H, cfg.inter), "lm_head": (cfg.vocab, H)}


@pytest.mark.parametrize("kw", [QWEN3_8B, LLAMA3_70B])
@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_tp_plan_partitions_every_projection(kw, size):
    cfg = cuda.synth_config(**kw, max_pos=64)
    shapes = full_shapes(cfg)
    plans = [cuda.tp_plan(cfg, r, size) for r in range(size)]
    for name, (rows, cols) in shapes.items():
        cover = np.zeros((rows, cols // 64), np.int32)   # in groups of 64 columns
        for p in plans:
            r0, nr, c0, nc = p[name]
            assert c0 % 64 == 0 and nc % 64 == 0, (name, p[name])   # group boundaries
            assert nr % 16 == 0                                        # whole row blocks
            cover[r0:r0 + nr, c0 // 64:(c0 + nc) // 64] += 1
        assert np.all(cover == 1), name


def test_tp_plan_rejects_indivisible_degree():
    cfg = cuda.synth_config(**QWEN3_8B, max_pos=64)
    with pytest.raises(cuda.CudaError):
        cuda.tp_plan(cfg, 0, 3)


def dequant(w, s, b, G):
    rows, cols8 = w.shape
    q = ((w[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(rows, cols8 * 8)
    sf = np.repeat(s, G, axis=1)
    bf = np.repeat(b, G, axis=1)
    return (sf * q + bf).astype(np.float32)


def layer_mats(cfg, seed):
    rng = np.random.default_rng(seed)
    mats = {}
    for name, (rows, cols) in full_shapes(cfg).items():
        if name == "lm_head":
            continue
        w = rng.integers(0, 2**32, (rows, cols // 8), dtype=np.uint64).astype(np.uint32)
        s = rng.uniform(0.001, 0.01, (rows, cols // 64)).astype(np.float32)
        b = rng.uniform(-0.05, 0.05, (rows, cols // 64)).astype(np.float32)
        mats[name] = dequant(w, s, b, 64)
    return mats


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


SMALL = dict(hidden=512, layers=1, n_heads=8, n_kv_heads=4, head_dim=64, inter=1024, vocab=1024, tie=False)


def _rank_main(rank, size, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    import torch
    try:
        cfg = cuda.synth_config(**SMALL, max_pos=64)
        plan = cuda.tp_plan(cfg, rank, size)
        mats = layer_mats(cfg, seed=7)   # every rank holds the same checkpoint
        rng = np.random.default_rng(11)
        x = rng.standard_normal(cfg.hidden).astype(np.float32)
        att = rng.standard_normal(cfg.n_heads * cfg.head_dim).astype(np.float32)
        act = rng.standard_normal(cfg.inter).astype(np.float32)
        res = {}
        # column-parallel: this rank's rows, gathered in rank order
        for name in ("q", "k", "v", "gate", "up"):
            r0, nr, c0, nc = plan[name]
            y = torch.from_numpy(mats[name][r0:r0 + nr, c0:c0 + nc] @ x[c0:c0 + nc])
            parts = [torch.zeros_like(y) for _ in range(size)]
            dist.all_gather(parts, y)
            res[name] = torch.cat(parts).numpy()
        # row-parallel: f32 partial over this rank's columns, summed over ranks
        for name, xin in (("o", att), ("down", act)):
            r0, nr, c0, nc = plan[name]
            p = torch.from_numpy(mats[name][r0:r0 + nr, c0:c0 + nc] @ xin[c0:c0 + nc])
            dist.all_reduce(p)
            res[name] = p.numpy()
        import bench
        res["max"] = bench.max_over_ranks(dist, [rank + 1.0, 10.0 - rank])
        if rank == 0:
            full = {n: mats[n] @ x for n in ("q", "k", "v", "gate", "up")}
            full["o"] = mats["o"] @ att
            full["down"] = mats["down"] @ act
            err = {n: float(np.abs(res[n] - full[n]).max() / max(1e-6, np.abs(full[n]).max()))
                   for n in full}
            out.put((err, res["max"]))
    finally:
        dist.destroy_process_group()


def test_tp_world2_shards_reproduce_the_full_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, mx = q.get(timeout=10)
    # gathers are exact; the all-reduce adds two f32 partials (order differs)
    for n, e in err.items():
        assert e < 1e-5, (n, e)
    assert mx == [2.0, 10.0]
