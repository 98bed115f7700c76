"""Tensor parallel on 2, 4 or 8 GPUs (each size skipped with fewer): a small
synthetic Qwen3-architecture model sharded over the ranks (one process per
GPU, NCCL communicator and NVLink mailboxes bound through the C ABI) against
the oracle, which runs the unsharded model.

The row-parallel projections (o_proj, down_proj) leave exact f64 partials of
the projection arithmetic; the one-token step adds them in rank order inside
its own exchange kernel, so the sharded model gives the oracle's logits bit
for bit, and its greedy and sampled tokens. A second test holds one rank back
and checks that the other's bounded wait ends the step with an error instead
of hanging, and that its CUDA context stays usable."""
import os
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from mlxd_b200 import cuda
from oracle import pyoracle as po
from tests.helpers import bf16_to_f32, orc_config

pytestmark = pytest.mark.gpu

KW = dict(hidden=512, layers=3, n_heads=16, n_kv_heads=8, head_dim=64, inter=1024, vocab=4096,
          max_pos=256)
SAMPLED = dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1, repetition_context=16,
               seed=4)


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _ids():
    return np.random.default_rng(5).integers(0, KW["vocab"], 24).tolist()


def _join(uid_q, rank, size):
    if rank == 0:
        uid = np.zeros(128, np.uint8)
        cuda.check(cuda.lib().mlxd_cuda_nccl_unique_id(cuda.ptr(uid)), "nccl id")
        for _ in range(size - 1):
            uid_q.put(uid.tobytes())
        return uid.tobytes()
    return uid_q.get(timeout=120)


def _model(rank, size):
    cuda.init(rank)
    cfg = cuda.synth_config(**KW, tp_rank=rank, tp_size=size)
    host = cuda.synth_host_tensors(cuda.synth_config(**KW), seed=3)
    return cuda.Model(cfg, host)


def _rank_parity(rank, size, uid_q, out_q):
    m = _model(rank, size)
    m.tp_init(_join(uid_q, rank, size))
    ids = _ids()
    kv = m.new_kv(64)
    m.forward(kv, ids[:20], want_logits=False)          # chunk kernels, NCCL partial sums
    logits = [np.asarray(m.forward(kv, [t])) for t in ids[20:]]   # one-token steps
    greedy = m.generate(ids[:16], 24)[0]
    sampled, slp, _ = m.generate(ids[:16], 24, sp=cuda.sampling(**SAMPLED), logprobs=True)
    glp_toks, glp, _ = m.generate(ids[:16], 12, logprobs=True)
    out_q.put((rank, logits, np.asarray(greedy), np.asarray(sampled), np.asarray(slp),
               np.asarray(glp_toks), np.asarray(glp)))
    m.close()


def _spawn(target, size, extra=()):
    """Start one process per rank. Returns the processes and the queues: the
    caller keeps every queue referenced until the ranks are done (a queue
    that is garbage-collected unlinks its semaphore, and a rank still
    starting up then fails to open it)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, size, uid_q, out_q) + tuple(extra)) for r in range(size)]
    for p in procs:
        p.start()
    return procs, out_q, uid_q


def _get(q, procs, timeout):
    """The next result, failing early when a rank has exited with an error."""
    t_end = time.time() + timeout
    while time.time() < t_end:
        try:
            return q.get(timeout=2)
        except Exception:
            bad = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if bad:
                for p in procs:
                    if p.exitcode is None:
                        p.kill()
                raise AssertionError("a rank exited with %s" % bad)
    raise AssertionError("no result within %d s" % timeout)


def _finish(procs):
    for p in procs:
        p.join(timeout=180)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(c == 0 for c in codes), codes


@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_matches_oracle_bit_exact(size):
    if _gpu_count() < size:
        pytest.skip(f"needs {size} GPUs")
    procs, out_q, uid_q = _spawn(_rank_parity, size)
    res = {}
    for _ in range(size):
        r, *rest = _get(out_q, procs, 600)
        res[r] = rest
    _finish(procs)
    cfg = cuda.synth_config(**KW)
    o = po.Oracle(orc_config(cfg), cuda.synth_host_tensors(cfg, seed=3))
    ids = _ids()
    okv = o.new_kv(64)
    o.forward(okv, ids[:20], want_logits=False)
    Vl = KW["vocab"] // size
    for i, t in enumerate(ids[20:]):
        ol = o.forward(okv, [t])
        tp = np.concatenate([bf16_to_f32(res[r][0][i]) for r in range(size)])
        assert tp.shape == (size * Vl,)
        assert np.array_equal(tp.view(np.uint32), np.asarray(ol, np.float32).view(np.uint32)), i
    og = o.generate(ids[:16], 24)[0]
    os_, olp, _ = o.generate(ids[:16], 24, sp=po.sampling(**SAMPLED))
    og12, oglp, _ = o.generate(ids[:16], 12)
    for r in range(size):
        greedy, sampled, slp, gt, glp = res[r][1:]
        assert np.array_equal(greedy, og), r
        assert np.array_equal(sampled, os_), r
        assert np.abs(slp - olp).max() < 1e-4, r
        assert np.array_equal(gt, og12), r
        assert np.abs(glp - oglp).max() < 1e-4, r


def _rank_stall(rank, size, uid_q, out_q, go_q):
    m = _model(rank, size)
    m.tp_init(_join(uid_q, rank, size))
    if rank == 0:
        # rank 1 never runs this step: every exchange waits out its limit
        kv = m.new_kv(8)
        t0 = time.time()
        msg = ""
        try:
            m.forward(kv, [7])
        except cuda.CudaError as e:
            msg = str(e)
        dt = time.time() - t0
        # the context still works: a projection after the failed step
        rng = np.random.default_rng(0)
        w = rng.integers(0, 2**32, (64, 8), dtype=np.uint64).astype(np.uint32)
        s = np.full((64, 1), 0x3C00, np.uint16)
        b = np.zeros((64, 1), np.uint16)
        lin = cuda.Linear(w, s, b, 64)
        y = lin(np.full(64, 0x3F80, np.uint16))
        cuda.synchronize()
        out_q.put((msg, dt, int(np.asarray(y).view(np.uint16).any())))
        lin.close()
        go_q.put(1)
    else:
        go_q.get(timeout=300)
    m.close()


def test_tp_peer_that_never_arrives_fails_the_step():
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    go_q = ctx.Queue()
    procs, out_q, uid_q = _spawn(_rank_stall, 2, (go_q,))
    msg, dt, ok = _get(out_q, procs, 300)
    _finish(procs)
    assert "gave up waiting for a peer GPU" in msg, msg
    # six exchanges (two per layer), each giving up after about a second
    assert 2.0 < dt < 60.0, dt
    assert ok
