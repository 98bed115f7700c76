"""The CPU oracle pinned against the reference's own golden vectors and
known-answer tests (tests/golden/goldens.json, copied from the reference's
test sources by tests/golden/make_fixtures.py), plus the self-consistency
properties the reference tests (incremental == full, chunked == full, window
semantics). CPU only."""
import math
import os

import numpy as np
import pytest

from oracle import pyoracle as po

K_LOGITS = np.array([0.1, -2.0, 3.5, 1.0, 0.0, 2.9, -1.0, 0.5], np.float32)


def fixture(golden_dir, name):
    return os.path.join(golden_dir, name)


# ---- G1: greedy sequence (tests/test_engine_gpu.c:21-23, :157-228)

def test_kOracle_greedy_tiny_qwen3(golden_dir, goldens):
    g = goldens["kOracle"]
    o = po.Oracle.from_dir(fixture(golden_dir, g["fixture"]))
    toks, _, margins = o.generate(g["prompt"], g["max_tokens"])
    assert list(map(int, toks)) == g["ids"]
    # the pin is sharp: two steps are decided by one bf16 ulp
    assert float(margins.min()) <= 0.0021


def test_generate_deterministic(golden_dir, goldens):
    o = po.Oracle.from_dir(fixture(golden_dir, "tiny_qwen3"))
    a, _, _ = o.generate([1, 2], 8)
    b, _, _ = o.generate([1, 2], 8)
    assert np.array_equal(a, b)


# ---- G2/G3: qwen3_5 logits (tests/test_qwen3_5_goldens_gpu.c:14-30, 119-129)

@pytest.mark.parametrize("key", ["qwen3_5_dense", "qwen3_5_tied"])
def test_qwen3_5_first8_logits(golden_dir, goldens, key):
    g = goldens[key]
    o = po.Oracle.from_dir(fixture(golden_dir, g["fixture"]))
    kv = o.new_kv(16)
    lg = o.forward(kv, g["ids"])
    assert int(np.argmax(lg)) == g["argmax"]
    assert np.abs(lg[:8] - np.array(g["first8"])).max() <= g["atol"]


# ---- G4: llama3 RoPE frequencies (tests/test_rope_llama3.c:173-224)

def test_llama3_freq_golden(golden_dir, goldens):
    import json
    g = goldens["llama3_freqs"]
    cj = json.load(open(os.path.join(golden_dir, g["config"], "config.json")))
    rs = cj["rope_scaling"]
    hd = cj["hidden_size"] // cj["num_attention_heads"]
    assert hd == g["head_dim"]
    fr = po.llama3_freqs(cj["rope_theta"], rs["factor"], rs["low_freq_factor"],
                         rs["high_freq_factor"], rs["original_max_position_embeddings"], hd)
    gold = np.array(g["freqs"], np.float64)
    rel = np.abs(fr - gold) / np.abs(gold)
    assert rel.max() < g["rtol"]
    # dim 29, smooth band (tests/test_rope_llama3.c:165-169)
    assert abs(fr[29] - 4.61558892e+02) / 4.61558892e+02 < 1e-5


@pytest.mark.parametrize("args", [(5e5, 0.0, 1.0, 4.0, 8192), (5e5, -1.0, 1.0, 4.0, 8192),
                                  (5e5, 8.0, 1.0, 1.0, 8192), (5e5, 8.0, 1.0, 4.0, 0)])
def test_llama3_freq_rejects(args):
    with pytest.raises(ValueError):
        po.llama3_freqs(*args, 128)


# ---- G5: sampler known answers (tests/test_sampler_gpu.c:19-522)

def test_sampler_greedy():
    tok, lp, keep = po.sample(K_LOGITS, po.sampling(temperature=0.0))
    assert tok == 2 and keep.sum() == 1


def test_top_k_filter():
    out = po.top_k(K_LOGITS, 3)
    for i in range(8):
        if i in (2, 5, 3):
            assert out[i] == K_LOGITS[i]
        else:
            assert np.isneginf(out[i])
    for k in (-1, 8, 13):
        assert np.array_equal(po.top_k(K_LOGITS, k), K_LOGITS)


def test_top_k1_equals_greedy():
    for step in range(16):
        tok, _, _ = po.sample(K_LOGITS, po.sampling(temperature=5.0, top_k=1), step=step)
        assert tok == 2


def test_top_p_filter():
    vals = np.log(np.array([0.15, 0.5, 0.05, 0.3], np.float32))
    out = po.top_p(vals, 0.7)
    assert np.isneginf(out[0]) and np.isneginf(out[2])
    assert abs(out[1] - vals[1]) < 1e-6 and abs(out[3] - vals[3]) < 1e-6
    assert np.allclose(po.top_p(vals, 1.0), vals)


def test_top_p_zero_is_greedy():
    out = po.top_p(K_LOGITS, 0.0)
    assert out[2] == K_LOGITS[2] and np.isneginf(np.delete(out, 2)).all()
    for step in range(16):
        tok, _, _ = po.sample(K_LOGITS, po.sampling(temperature=5.0, top_p=0.0), step=step)
        assert tok == 2


def test_top_p_tiny_p_never_empty():
    uni = np.zeros(8, np.float32)
    assert np.array_equal(po.top_p(uni, 1e-9), uni)
    out = po.top_p(K_LOGITS, 1e-9)
    assert out[2] == K_LOGITS[2] and np.isneginf(np.delete(out, 2)).all()


def test_min_p_filter():
    out = po.min_p(K_LOGITS, 0.5)
    for i in range(8):
        if i in (2, 5):
            assert out[i] == K_LOGITS[i]
        else:
            assert np.isneginf(out[i])
    assert np.array_equal(po.min_p(K_LOGITS, 0.0), K_LOGITS)


def test_seeded_reproducibility():
    uni = np.array([0.0, 0.01, -0.01, 0.02, -0.02, 0.03, -0.03, 0.015], np.float32)
    sp = po.sampling(temperature=1.0, seed=42)
    a = [po.sample(uni, sp, step=i)[0] for i in range(16)]
    b = [po.sample(uni, sp, step=i)[0] for i in range(16)]
    c = [po.sample(uni, po.sampling(temperature=1.0, seed=7), step=i)[0] for i in range(16)]
    assert a == b and a != c and len(set(a)) > 1


def test_logprob_from_raw_logits():
    mx = K_LOGITS.max()
    lse = mx + math.log(np.exp(K_LOGITS.astype(np.float64) - mx).sum())
    want = K_LOGITS[2] - lse
    for sp in (po.sampling(temperature=0.7, top_k=1), po.sampling(temperature=0.0)):
        tok, lp, _ = po.sample(K_LOGITS, sp)
        assert tok == 2 and abs(lp - want) < 1e-4


@pytest.mark.parametrize("min_p,allowed", [(0.1, {2, 5, 3}), (0.35, {2, 5})])
def test_combined_filters(min_p, allowed):
    sp = po.sampling(temperature=2.0, top_k=4, top_p=0.9, min_p=min_p, seed=77)
    seen = set()
    for step in range(32):
        tok, _, keep = po.sample(K_LOGITS, sp, step=step)
        assert tok in allowed
        assert set(np.nonzero(keep)[0].tolist()) == allowed
        seen.add(tok)
    assert len(seen) >= 2


def test_repetition_penalty_rule():
    # build-defined (mlx-lm rule): x>0 -> x/p, x<=0 -> x*p over distinct recent ids
    x = np.array([2.0, -1.0, 0.5, 3.0], np.float32)
    sp = po.sampling(temperature=1.0, top_k=1, repetition_penalty=2.0, repetition_context=2)
    tok, _, _ = po.sample(x, sp, ctx=np.array([3, 3], np.int32))
    assert tok == 0          # 3.0 -> 1.5 < 2.0
    tok, _, _ = po.sample(x, sp, ctx=np.array([3, 0, 1], np.int32))
    assert tok == 3          # only the last two ids (0, 1) are penalised


def test_own_exp_accuracy():
    xs = np.linspace(-100, 80, 20001, dtype=np.float32)
    L = po.lib()
    got = np.array([L.orc_expf(float(v)) for v in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    normal = xs >= -87.0
    rel = np.abs(got - ref)[normal] / ref[normal]
    assert rel.max() < 4e-7
    assert np.abs(got - ref)[~normal].max() < 1e-38    # subnormal results
    assert L.orc_expf(float("-inf")) == 0.0


# ---- G6: quantized matmul KAT (tests/test_mlxbridge_gpu.c:563-642)

def test_qmm_kat_mean_480():
    w = (np.arange(8 * 64) % 16).astype(np.float32).reshape(8, 64)
    wq, s, b = po.affine_quantize(w, 64)
    deq = np.zeros_like(w)
    for r in range(8):
        for j in range(64):
            q = (int(wq[r, j // 8]) >> (4 * (j % 8))) & 0xF
            deq[r, j] = s[r, j // 64] * q + b[r, j // 64]
    assert np.abs(deq - w).max() < 0.01
    x = po.f32_to_bf16(np.ones(64, np.float32))
    for exact in (True, False):
        y = po.bf16_to_f32(po.qlinear(x, wq, s, b, 64, exact=exact))
        assert y.shape == (1, 8)
        assert abs(float(y.mean()) - 480.0) < 1.0


def test_quantize_nibble_order_lsb_first():
    w = np.zeros((1, 64), np.float32)
    w[0, 1] = 15.0     # element 1 -> word 0, nibble 1
    w[0, 9] = 15.0     # element 9 -> word 1, nibble 1
    wq, s, b = po.affine_quantize(w, 64)
    q = [(int(wq[0, j // 8]) >> (4 * (j % 8))) & 0xF for j in range(64)]
    lv = [q[1], q[9]]
    assert lv[0] == lv[1] and all(q[j] != lv[0] for j in range(64) if j not in (1, 9))


# ---- G7: sliding-window mask KAT (tests/test_forward_d0_gpu.c:829-905)

def test_window_mask_kat():
    m = po.window_mask(3, 5, 2).astype(int)
    assert m.tolist() == [[0, 1, 1, 0, 0], [0, 0, 1, 1, 0], [0, 0, 0, 1, 1]]
    d = po.window_mask(1, 5, 2).astype(int)
    assert d.tolist() == [[0, 0, 0, 1, 1]]
    assert po.window_mask(1, 2, 4).all()
    with pytest.raises(ValueError):
        po.window_mask(5, 3, 2)


# ---- self-consistency (tests/test_forward_gpu.c:615-864)

@pytest.mark.parametrize("name,tol", [("tiny_qwen3", 5e-2), ("tiny_qwen3_tied", 0.1)])
def test_incremental_equals_full(golden_dir, name, tol):
    o = po.Oracle.from_dir(fixture(golden_dir, name))
    ids = [5, 17, 3, 99]
    kv = o.new_kv(8)
    full = o.forward(kv, ids)
    kv2 = o.new_kv(8)
    o.forward(kv2, ids[:3], want_logits=False)
    inc = o.forward(kv2, ids[3:])
    assert int(np.argmax(full)) == int(np.argmax(inc))
    assert np.abs(full - inc).max() < tol


def test_chunked_prefill_equals_full(golden_dir):
    o = po.Oracle.from_dir(fixture(golden_dir, "tiny_qwen3"))
    ids = list(range(1, 11))
    kv = o.new_kv(16)
    full = o.forward(kv, ids)
    kv2 = o.new_kv(16)
    o.forward(kv2, ids[:4], want_logits=False)
    o.forward(kv2, ids[4:7], want_logits=False)
    ch = o.forward(kv2, ids[7:])
    assert int(np.argmax(full)) == int(np.argmax(ch))
    assert np.abs(full - ch).max() < 5e-2


def test_causal_probe(golden_dir):
    o = po.Oracle.from_dir(fixture(golden_dir, "tiny_qwen3"))
    a = o.forward_hidden(o.new_kv(8), [1, 2, 3])
    b = o.forward_hidden(o.new_kv(8), [1, 2, 77])
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert not np.array_equal(a[2], b[2])


def _mistral_pair(golden_dir, name):
    import json
    d = fixture(golden_dir, name)
    cj = json.load(open(os.path.join(d, "config.json")))
    t = po.read_checkpoint(d)
    win = po.Oracle(po.config_from_json(cj), t)
    cj2 = dict(cj)
    cj2["sliding_window"] = None
    nowin = po.Oracle(po.config_from_json(cj2), t)
    return win, nowin, cj["sliding_window"]


@pytest.mark.parametrize("name", ["tiny_mistral", "tiny_mistral_tied"])
def test_window_within_and_beyond(golden_dir, name):
    win, nowin, W = _mistral_pair(golden_dir, name)
    assert W == 8
    rng = np.random.default_rng(0)
    for S in (1, W):
        ids = rng.integers(0, 256, S).tolist()
        a = win.forward(win.new_kv(16), ids)
        b = nowin.forward(nowin.new_kv(16), ids)
        assert np.abs(a - b).max() < 2e-3
    ids = rng.integers(0, 256, W + 2).tolist()
    a = win.forward(win.new_kv(16), ids)
    b = nowin.forward(nowin.new_kv(16), ids)
    assert np.abs(a - b).max() > 1e-2


def test_window_boundary_incremental_equals_full(golden_dir):
    win, _, W = _mistral_pair(golden_dir, "tiny_mistral")
    ids = list(range(3, 3 + W + 3))
    full = win.forward(win.new_kv(32), ids)
    kv = win.new_kv(32)
    win.forward(kv, ids[:-1], want_logits=False)
    inc = win.forward(kv, ids[-1:])
    assert int(np.argmax(full)) == int(np.argmax(inc))
    assert np.abs(full - inc).max() < 5e-2


def test_context_overflow_rejected(golden_dir):
    o = po.Oracle.from_dir(fixture(golden_dir, "tiny_qwen3_5"))   # max_pos 512
    with pytest.raises(RuntimeError):
        o.generate(list(range(1, 200)) * 3, 2)
