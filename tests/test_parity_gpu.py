"""GPU parity: every kernel path of libmlxd_cuda against the CPU oracle, called
through the C ABI, on the reference's fixtures and on seeded synthetic
models. The library and the oracle compute projections and attention with
one specified arithmetic (per-group fixed-point inputs with exact integer
group sums and f64 combination, rounded once; attention in fixed blocks of
64 positions with f64 merges), so the bar is identical bits: logits, KV
cache rows and greedy tokens. Where a test states a tolerance instead, it is
the north-star bound (max-abs 2e-2, mean-abs relative 1e-3) and the test
says why."""
import os

import numpy as np
import pytest

from mlxd_b200 import cuda
from oracle import pyoracle as po
from tests.helpers import bf16_to_f32, f32_to_bf16, logits_close, orc_config, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    cuda.init(0)
    yield


def same_bits(g, o):
    """bf16 arrays (uint16 bits or their f32 values) identical, NaN-free."""
    g, o = np.asarray(g), np.asarray(o)
    return g.shape == o.shape and np.array_equal(g, o)


# ------------------------------------------------------------- projections

def synth_triplet(rows, cols, group, seed, f32_scales=False, std=0.02):
    w = np.zeros((rows, cols // 8), np.uint32)
    s = np.zeros((rows, cols // group), np.uint16)
    b = np.zeros((rows, cols // group), np.uint16)
    cuda.lib().mlxd_host_synth_quantized(cuda.ptr(w), cuda.ptr(s), cuda.ptr(b), rows, cols,
                                         group, seed, std)
    if f32_scales:
        return w, bf16_to_f32(s).copy(), bf16_to_f32(b).copy()
    return w, s, b


# (rows, cols, group, f32 scales): the Qwen3-8B projection shapes on the
# integer-MMA decode kernel, a vocabulary-sized one, and the generic kernel's
# formats (group 32, f32 scales, widths that are not multiples of 512)
GEMV_SHAPES = [(256, 512, 64, False), (4096, 4096, 64, False), (1024, 4096, 64, False),
               (24576, 4096, 64, False), (4096, 12288, 64, False), (151936, 1024, 64, False),
               (96, 64, 32, True), (128, 128, 32, False), (64, 192, 64, True), (256, 320, 64, False)]


def input_vector(cols, rng, kind):
    if kind == "normal":
        return rand_bf16(cols, rng)
    if kind == "wide":
        # magnitudes over 40 binades, zeros, and a few tiny values in a group
        # with a large one: the fixed point's rounding of small inputs
        x = rng.standard_normal(cols).astype(np.float32) * np.exp2(rng.integers(-30, 10, cols)).astype(np.float32)
        x[rng.integers(0, cols, cols // 16)] = 0.0
        return f32_to_bf16(x)
    # SwiGLU-like: many near-zero values
    g = rng.standard_normal(cols).astype(np.float32) * 2
    u = rng.standard_normal(cols).astype(np.float32)
    return f32_to_bf16(g / (1 + np.exp(-g)) * u)


@pytest.mark.parametrize("rows,cols,group,f32", GEMV_SHAPES)
@pytest.mark.parametrize("kind", ["normal", "wide", "act"])
def test_decode_gemv_bit_exact(rows, cols, group, f32, kind):
    rng = np.random.default_rng(rows + cols)
    w, s, b = synth_triplet(rows, cols, group, rows * 7 + cols, f32)
    x = input_vector(cols, rng, kind)
    lin = cuda.Linear(w, s, b, group)
    g = lin(x)[0]
    o = po.qlinear(x, w, s, b, group, exact=True)[0]
    assert same_bits(g, o), int(np.sum(g != o))


@pytest.mark.parametrize("S", [2, 5, 64, 130])
@pytest.mark.parametrize("rows,cols,group,f32", [(256, 512, 64, False), (96, 64, 32, True),
                                                 (1024, 1024, 64, False), (512, 4096, 64, False)])
def test_prefill_gemm_bit_exact(S, rows, cols, group, f32):
    """A chunk of tokens gives the oracle's bits, and each row the bits the
    one-token kernel gives for it."""
    rng = np.random.default_rng(S * 31 + rows)
    w, s, b = synth_triplet(rows, cols, group, S + rows, f32)
    x = rand_bf16((S, cols), rng)
    lin = cuda.Linear(w, s, b, group)
    g = lin(x)
    o = po.qlinear(x, w, s, b, group, exact=True)
    assert same_bits(g, o), int(np.sum(g != o))
    for r in (0, S // 2, S - 1):
        assert same_bits(lin(x[r])[0], g[r])


@pytest.mark.parametrize("rows,n", [(1, 64), (7, 1024), (3, 4096), (5, 128), (2, 300)])
def test_rmsnorm_bit_exact(rows, n):
    rng = np.random.default_rng(n)
    x = rand_bf16((rows, n), rng, 3.0)
    w = rand_bf16(n, rng)
    assert np.array_equal(cuda.rmsnorm(x, w, 1e-6), po.rmsnorm(x, w, 1e-6))


# ------------------------------------------------------------------ sampler

K_LOGITS = np.array([0.1, -2.0, 3.5, 1.0, 0.0, 2.9, -1.0, 0.5], np.float32)


def test_sampler_kats_on_gpu():
    """The reference's sampler known answers (tests/test_sampler_gpu.c)."""
    sp = cuda.sampling
    assert cuda.sample(K_LOGITS, sp(temperature=0.0))[0] == 2
    for step in range(8):
        assert cuda.sample(K_LOGITS, sp(temperature=5.0, top_k=1), step=step)[0] == 2
        assert cuda.sample(K_LOGITS, sp(temperature=5.0, top_p=0.0), step=step)[0] == 2
    vals = np.log(np.array([0.15, 0.5, 0.05, 0.3], np.float32))
    keep = cuda.sample(vals, sp(temperature=1.0, top_p=0.7))[2]
    assert set(np.nonzero(keep)[0].tolist()) == {1, 3}
    keep = cuda.sample(K_LOGITS, sp(temperature=1.0, min_p=0.5))[2]
    assert set(np.nonzero(keep)[0].tolist()) == {2, 5}
    keep = cuda.sample(np.zeros(8, np.float32), sp(temperature=1.0, top_p=1e-9))[2]
    assert keep.all()
    for min_p, allowed in ((0.1, {2, 5, 3}), (0.35, {2, 5})):
        for step in range(16):
            tok, _, keep = cuda.sample(K_LOGITS, sp(temperature=2.0, top_k=4, top_p=0.9,
                                                    min_p=min_p, seed=77), step=step)
            assert tok in allowed and set(np.nonzero(keep)[0].tolist()) == allowed
    mx = K_LOGITS.max()
    want = K_LOGITS[2] - (mx + np.log(np.exp(K_LOGITS.astype(np.float64) - mx).sum()))
    # logprob from the raw logits (sampler.c:315-322): f32 logsumexp, 1e-4
    assert abs(cuda.sample(K_LOGITS, sp(temperature=0.0))[1] - want) < 1e-4
    assert abs(cuda.sample(K_LOGITS, sp(temperature=0.7, top_k=1))[1] - want) < 1e-4


SAMPLER_CASES = [
    dict(temperature=0.0),
    dict(temperature=0.0, repetition_penalty=1.3),
    dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1, seed=5),
    dict(temperature=1.0, top_p=0.9, seed=9),
    dict(temperature=0.8, min_p=0.05, seed=3),
    dict(temperature=1.3, top_k=1000, top_p=0.5, min_p=0.01, seed=11),
    dict(temperature=0.6, top_k=20, seed=2),
]


@pytest.mark.parametrize("case", range(len(SAMPLER_CASES)))
@pytest.mark.parametrize("V", [151936, 32768, 256])
def test_sampler_sets_and_draws_bit_exact(case, V):
    """Candidate index sets are bit-exact given identical logits; draws too
    (same uniform stream and association); logprob within 1e-4."""
    rng = np.random.default_rng(case * 100 + V)
    logits = f32_to_bf16(rng.standard_normal(V).astype(np.float32) * 3.0)
    lf = bf16_to_f32(logits)
    sp = cuda.sampling(**SAMPLER_CASES[case])
    osp = po.sampling(**SAMPLER_CASES[case])
    # context ids that include the current argmax, so the penalty moves it
    ctx = np.concatenate([rng.integers(0, V, 39), [int(np.argmax(lf))]]).astype(np.int32)
    for step in range(3):
        gt, glp, gk = cuda.sample(logits, sp, ctx=ctx, step=step)
        ot, olp, ok = po.sample(lf, osp, ctx=ctx, step=step)
        assert np.array_equal(gk, ok), (int(gk.sum()), int(ok.sum()))
        assert gt == ot
        assert abs(glp - olp) < 1e-4


@pytest.mark.parametrize("V,ties", [(151936, 5000), (32768, 4200)])
def test_sampler_top_k_with_ties_past_the_candidate_list(V, ties):
    """A top-k cut whose cutoff value is shared by more logits than the
    candidate list holds (4096): every tie survives (mlx keeps values >= the
    k-th largest) and the draw is still the oracle's."""
    rng = np.random.default_rng(V)
    lf = np.full(V, -3.0, np.float32)
    idx = rng.permutation(V)
    lf[idx[:10]] = rng.uniform(2.0, 5.0, 10).astype(np.float32)
    lf[idx[10:10 + ties]] = 1.0
    logits = f32_to_bf16(lf)
    lf = bf16_to_f32(logits)
    for kw in (dict(temperature=0.7, top_k=50, seed=3), dict(temperature=1.0, top_k=20, top_p=0.95, seed=8)):
        sp, osp = cuda.sampling(**kw), po.sampling(**kw)
        for step in range(3):
            gt, glp, gk = cuda.sample(logits, sp, step=step)
            ot, olp, ok = po.sample(lf, osp, step=step)
            assert int(gk.sum()) >= ties and np.array_equal(gk, ok)
            assert gt == ot and abs(glp - olp) < 1e-4


# ---------------------------------------------------------- whole forwards

def fixture_models(golden_dir, name):
    d = os.path.join(golden_dir, name)
    return cuda.Model.from_dir(d), po.Oracle.from_dir(d)


def test_kOracle_greedy_on_gpu(golden_dir, goldens):
    g = goldens["kOracle"]
    m, _ = fixture_models(golden_dir, g["fixture"])
    toks, _, _ = m.generate(g["prompt"], g["max_tokens"])
    assert list(map(int, toks)) == g["ids"]


@pytest.mark.parametrize("key", ["qwen3_5_dense", "qwen3_5_tied"])
def test_qwen3_5_goldens_on_gpu(golden_dir, goldens, key):
    """mlx-lm's logits (tests/test_qwen3_5_goldens_gpu.c: atol 1e-2 bf16,
    5e-2 4-bit) and the oracle's bits."""
    g = goldens[key]
    m, o = fixture_models(golden_dir, g["fixture"])
    lg = bf16_to_f32(m.forward(m.new_kv(16), g["ids"]))
    assert int(np.argmax(lg)) == g["argmax"]
    assert np.abs(lg[:8] - np.array(g["first8"])).max() <= g["atol"]
    ol = o.forward(o.new_kv(16), g["ids"])
    assert same_bits(lg, ol)


FIXTURES = ["tiny_qwen3", "tiny_qwen3_tied", "tiny_qwen3_5", "tiny_qwen3_5_tied", "tiny_llama3",
            "tiny_llama3_tied", "tiny_mistral", "tiny_mistral_tied"]


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_prefill_decode_vs_oracle(golden_dir, name):
    m, o = fixture_models(golden_dir, name)
    rng = np.random.default_rng(len(name))
    ids = rng.integers(0, 256, 13).tolist()
    kv, okv = m.new_kv(32), o.new_kv(32)
    for part in [ids[:9], ids[9:10], ids[10:12], ids[12:]]:
        assert same_bits(bf16_to_f32(m.forward(kv, part)), o.forward(okv, part))
    assert kv.offset() == 13
    for layer in range(2):
        for value in (False, True):
            assert same_bits(kv.read(layer, value), okv.read(layer, value))


@pytest.mark.parametrize("name", ["tiny_qwen3", "tiny_qwen3_tied", "tiny_mistral_tied"])
def test_fixture_generate_matches_oracle(golden_dir, name):
    m, o = fixture_models(golden_dir, name)
    prompt = list(range(5, 21))
    gt, _, _ = m.generate(prompt, 32)
    ot, _, _ = o.generate(prompt, 32)
    assert np.array_equal(gt, ot)


# ------------------------------------------------- synthetic 4-bit models

def synth_pair(cfg, seed=1, std=0.02):
    host = cuda.synth_host_tensors(cfg, seed=seed, std=std)
    return cuda.Model(cfg, host), po.Oracle(orc_config(cfg), host)


def qwen3_small(**kw):
    base = dict(hidden=512, layers=3, n_heads=8, n_kv_heads=2, head_dim=128, inter=1024,
                vocab=4096, max_pos=512)
    base.update(kw)
    return cuda.synth_config(**base)


def test_fast_decode_path_logits_and_kv():
    """Prefill (chunk kernels) then the one-token decode kernels: logits and
    every KV row identical to the oracle's."""
    cfg = qwen3_small()
    m, o = synth_pair(cfg)
    rng = np.random.default_rng(0)
    ids = rng.integers(0, cfg.vocab, 140).tolist()
    kv, okv = m.new_kv(160), o.new_kv(160)
    m.forward(kv, ids[:133], want_logits=False)
    o.forward(okv, ids[:133], want_logits=False)
    for t in ids[133:]:
        assert same_bits(bf16_to_f32(m.forward(kv, [t])), o.forward(okv, [t]))
    for layer in range(cfg.layers):
        for value in (False, True):
            assert same_bits(kv.read(layer, value), okv.read(layer, value))


def test_incremental_equals_full_on_gpu():
    """Decode steps and one prefill chunk over the same positions give the
    same bits (attention in absolute 64-position blocks, one projection
    arithmetic): the reference's incremental == full test
    (tests/test_forward_gpu.c:615-790) at zero tolerance."""
    cfg = qwen3_small(layers=2)
    m, _ = synth_pair(cfg, seed=4)
    ids = cuda.synth_prompt(150, cfg.vocab, 8).tolist()
    ka, kb = m.new_kv(160), m.new_kv(160)
    full = m.forward(ka, ids)
    m.forward(kb, ids[:70], want_logits=False)
    for t in ids[70:-1]:
        m.forward(kb, [t], want_logits=False)
    inc = m.forward(kb, ids[-1:])
    assert same_bits(full, inc)
    for layer in range(cfg.layers):
        assert same_bits(ka.read(layer), kb.read(layer))


@pytest.mark.parametrize("family,kw", [(cuda.QWEN3, {}), (cuda.MISTRAL, dict(window=24)),
                                       (cuda.MISTRAL, dict(window=100)),
                                       (cuda.QWEN3, dict(n_kv_heads=8)),
                                       (cuda.QWEN3, dict(n_kv_heads=4)),
                                       (cuda.QWEN3, dict(n_heads=16, n_kv_heads=2)),
                                       (cuda.QWEN3, dict(head_dim=64, n_heads=8, n_kv_heads=1)),
                                       (cuda.QWEN3, dict(head_dim=64, n_heads=8, n_kv_heads=4)),
                                       (cuda.QWEN3, dict(kvcap=9000, max_pos=9000)),
                                       (cuda.QWEN3, dict(kvcap=9000, max_pos=9000, n_kv_heads=8)),
                                       (cuda.MISTRAL, dict(window=8500, max_pos=9000))])
def test_decode_attention_variants_bit_exact(family, kw):
    """The decode attention on a plain cache, wrapping sliding-window rings
    (positions spread over several CTAs), and 1, 2, 4 and 8 query heads per kv
    head at head dims 128 and 64; caches whose attended span exceeds the
    cluster inbox (more than 128 blocks) take the global path."""
    kw = dict(kw)
    kvcap = kw.pop("kvcap", None)
    cfg = qwen3_small(family=family, layers=2, **kw)
    m, o = synth_pair(cfg, seed=6)
    rng = np.random.default_rng(6)
    ids = rng.integers(0, cfg.vocab, 330).tolist()
    kv = m.new_kv(kvcap or (kw["window"] + 16 if kw.get("window") else 340))
    okv = o.new_kv(340)
    for a0 in range(0, 320, 16):
        m.forward(kv, ids[a0:a0 + 16], want_logits=False)
        o.forward(okv, ids[a0:a0 + 16], want_logits=False)
    for t in ids[320:]:
        assert same_bits(bf16_to_f32(m.forward(kv, [t])), o.forward(okv, [t]))


@pytest.mark.parametrize("family,kw", [
    (cuda.QWEN3, {}),
    (cuda.LLAMA, dict(theta=5e5, llama3=(8.0, 1.0, 4.0, 8192))),
    (cuda.QWEN3, dict(tie=True, n_kv_heads=8)),
    (cuda.MISTRAL, dict(window=32)),
])
def test_greedy_64_tokens_identical(family, kw):
    """Identical greedy sequences for 64 tokens on N(0, 0.02) weights."""
    cfg = qwen3_small(family=family, **kw)
    m, o = synth_pair(cfg, 3)
    prompt = cuda.synth_prompt(57, cfg.vocab, seed=1)
    gt, _, _ = m.generate(prompt, 64, chunk=16)
    ot, _, _ = o.generate(prompt, 64, chunk=16)
    assert len(gt) == len(ot) == 64
    assert np.array_equal(gt, ot)


def test_sliding_window_ring_matches_oracle():
    # window 24 with chunked prefill so the ring wraps several times
    cfg = qwen3_small(family=cuda.MISTRAL, window=24, layers=2)
    m, o = synth_pair(cfg, seed=5)
    rng = np.random.default_rng(4)
    ids = rng.integers(0, cfg.vocab, 90).tolist()
    kv = m.new_kv(24 + 16)        # ring: window + chunk
    okv = o.new_kv(128)           # oracle: dense cache, window by masking
    for a in range(0, 80, 16):
        m.forward(kv, ids[a:a + 16], want_logits=False)
        o.forward(okv, ids[a:a + 16], want_logits=False)
    for t in ids[80:]:
        assert same_bits(bf16_to_f32(m.forward(kv, [t])), o.forward(okv, [t]))
    assert kv.offset() == 90


def test_sampled_generate_matches_oracle_generate():
    """Sampled generation (the Mistral-style settings) against the oracle's
    generate loop: identical tokens (same logits, same candidate sets, same
    uniform stream) and logprobs within 1e-4."""
    cfg = qwen3_small(layers=2)
    m, o = synth_pair(cfg, seed=7)
    kw = dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1, repetition_context=16, seed=4)
    prompt = cuda.synth_prompt(20, cfg.vocab, 2)
    gt, glp, _ = m.generate(prompt, 24, sp=cuda.sampling(**kw), logprobs=True)
    ot, olp, _ = o.generate(prompt, 24, sp=po.sampling(**kw))
    assert np.array_equal(gt, ot)
    assert np.abs(glp - olp).max() < 1e-4


def test_sampled_generate_graph_matches_step_loop():
    """Sampled generation replays one captured decode step (forward, sampler
    with device-side context length and step, token append); the tokens and
    logprobs equal a loop of forward + mlxd_cuda_sample with the context list
    and step passed from the host. The same cache then serves a short and a
    longer generation (the context list is reallocated and the graph
    recaptured), each equal to the step loop."""
    cfg = qwen3_small(layers=2)
    m, _ = synth_pair(cfg, seed=7)
    sp = cuda.sampling(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1,
                       repetition_context=16, seed=4)

    def step_loop(prompt, n):
        kv = m.new_kv(len(prompt) + n + 1)
        m.forward(kv, prompt[:-1].tolist(), want_logits=False)
        ctx, t, out, outlp = list(prompt), int(prompt[-1]), [], []
        for e in range(n):
            tok, lp, _ = cuda.sample(m.forward(kv, [t]), sp, ctx=np.array(ctx, np.int32), step=e)
            out.append(tok)
            outlp.append(lp)
            ctx.append(tok)
            t = tok
        return np.array(out, np.int32), np.array(outlp, np.float32)

    prompt = cuda.synth_prompt(20, cfg.vocab, 2)
    toks, lps, _ = m.generate(prompt, 12, sp=sp, logprobs=True)
    ref_t, ref_lp = step_loop(prompt, 12)
    assert np.array_equal(toks, ref_t) and np.array_equal(lps, ref_lp)
    # one cache for both: short, then longer (context list grows)
    kv = m.new_kv(200)
    short, _, _ = m.generate(prompt[:8], 6, sp=sp, kv=kv)
    assert np.array_equal(short, step_loop(prompt[:8], 6)[0])
    long_prompt = cuda.synth_prompt(150, cfg.vocab, 3)
    longer, _, _ = m.generate(long_prompt, 30, sp=sp, kv=kv)
    assert np.array_equal(longer, step_loop(long_prompt, 30)[0])
    # and the short one again on the same cache (graph replayed from fresh counters)
    again, _, _ = m.generate(prompt[:8], 6, sp=sp, kv=kv)
    assert np.array_equal(again, short)


def test_greedy_with_repetition_penalty_matches_oracle():
    """The penalty applies before greedy draws too (mlx-lm's logits
    processors run before the argmax)."""
    cfg = qwen3_small(layers=2)
    m, o = synth_pair(cfg, seed=11)
    kw = dict(temperature=0.0, repetition_penalty=1.5, repetition_context=8)
    prompt = cuda.synth_prompt(12, cfg.vocab, 5)
    gt, _, _ = m.generate(prompt, 20, sp=cuda.sampling(**kw))
    ot, _, _ = o.generate(prompt, 20, sp=po.sampling(**kw))
    assert np.array_equal(gt, ot)


def test_edge_cases():
    cfg = qwen3_small(layers=1, max_pos=64)
    m, o = synth_pair(cfg)
    # single-token prompt: no prefill, seed forward only
    gt, _, _ = m.generate([7], 5)
    ot, _, _ = o.generate([7], 5)
    assert np.array_equal(gt, ot)
    # max_new = 1
    assert len(m.generate([7, 8, 9], 1)[0]) == 1
    # context longer than max_position_embeddings
    with pytest.raises(cuda.CudaError):
        m.generate(list(range(70)), 2)
    # token id out of range
    with pytest.raises(cuda.CudaError):
        m.forward(m.new_kv(8), [cfg.vocab])
    # KV capacity exceeded
    kv = m.new_kv(4)
    m.forward(kv, [1, 2, 3, 4], want_logits=False)
    with pytest.raises(cuda.CudaError):
        m.forward(kv, [5])


def test_eos_stops_generation():
    cfg = qwen3_small(layers=1)
    m0, o = synth_pair(cfg, seed=9)
    ot, _, _ = o.generate([1, 2, 3], 6)
    cfg.n_eos = 1
    cfg.eos[0] = int(ot[2])
    m, _ = synth_pair(cfg, seed=9)
    gt, _, _ = m.generate([1, 2, 3], 6)
    assert list(gt) == list(ot[:2])


def test_weight_and_kv_memory_accounting():
    cfg = qwen3_small(layers=2)
    m, _ = synth_pair(cfg)
    before = cuda.lib().mlxd_cuda_active_memory()
    kv = m.new_kv(100)
    after = cuda.lib().mlxd_cuda_active_memory()
    expect = 2 * cfg.layers * cfg.n_kv_heads * 100 * cfg.head_dim * 2
    assert after - before >= expect
    kv.close()
    assert cuda.lib().mlxd_cuda_active_memory() <= after - expect + 64


# ------------------------------------------------ the benchmark configurations

def baseline_pair(cfg, seed=0):
    """Full-size synthetic weights made on the GPU; the oracle gets the same
    bits through host memory."""
    dev = cuda.synth_device_tensors(cfg, seed=seed)
    host = cuda.device_tensors_to_host(dev)
    return cuda.Model(cfg, dev, on_device=True), po.Oracle(orc_config(cfg), host)


def run_config(cfg, prompt_len, new, chunk=512, seed=0):
    m, o = baseline_pair(cfg, seed)
    prompt = cuda.synth_prompt(prompt_len, cfg.vocab, seed=seed)
    gt, _, _ = m.generate(prompt, new, chunk=chunk)
    ot, _, _ = o.generate(prompt, new, chunk=chunk)
    # logits of the first decode position (after the prompt), both sides
    kv, okv = m.new_kv(prompt_len + 1), o.new_kv(prompt_len + 1)
    g = bf16_to_f32(m.forward(kv, prompt.tolist()))
    ol = o.forward(okv, prompt.tolist())
    ok, mx, mr = logits_close(g, ol, max_abs=2e-2, mean_rel=1e-3)
    return gt, ot, g, ol, (ok, mx, mr)


def test_config_c1_tiny_qwen3_g64():
    """C1 exactly: 2 layers, hidden 64, 4/2 heads, head dim 16, MLP 128,
    vocab 256, tied, RMSNorm eps 1e-6, QK-norm, theta 1e6, 4-bit g64 bf16
    scales on N(0, 0.02); 16 prompt ids then 32 greedy tokens."""
    cfg = cuda.synth_config(hidden=64, layers=2, n_heads=4, n_kv_heads=2, head_dim=16, inter=128,
                            vocab=256, tie=True, max_pos=256)
    gt, ot, g, ol, (ok, mx, mr) = run_config(cfg, 16, 32)
    assert np.array_equal(gt, ot) and len(gt) == 32
    assert same_bits(g, ol) and ok


def test_config_c2_qwen3_0_6b():
    """C2: Qwen3-0.6B architecture, 512 prompt ids then 64 greedy tokens."""
    cfg = cuda.synth_config(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, inter=3072,
                            vocab=151936, tie=True, max_pos=40960)
    gt, ot, g, ol, (ok, mx, mr) = run_config(cfg, 512, 64)
    assert np.array_equal(gt, ot) and len(gt) == 64
    assert same_bits(g, ol) and ok


def test_config_c3_qwen3_8b_shortened():
    """C3 shortened: Qwen3-8B architecture, 128 prompt ids then 64 greedy
    tokens (the oracle decodes the 8B model at a few tokens per second)."""
    cfg = cuda.synth_config(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                            vocab=151936, max_pos=40960)
    gt, ot, g, ol, (ok, mx, mr) = run_config(cfg, 128, 64)
    assert np.array_equal(gt, ot) and len(gt) == 64
    assert same_bits(g, ol) and ok


def test_config_c4_mistral_window_shortened():
    """C4 shortened to 2 layers: Mistral-7B width (hidden 4096, 32/8 heads,
    head dim 128, MLP 14336, vocab 32768), sliding window 4096 over a ring of
    4607 slots, an 8192-token prompt in 512-token chunks (the ring wraps
    twice), then 48 sampled tokens at temperature 0.7, top-k 50, top-p 0.9,
    repetition penalty 1.1 over the last 256 tokens. The oracle keeps a dense
    cache and masks the window: identical tokens, logprobs within 1e-4."""
    cfg = cuda.synth_config(hidden=4096, layers=2, n_heads=32, n_kv_heads=8, head_dim=128, inter=14336,
                            vocab=32768, family=cuda.MISTRAL, window=4096, max_pos=8192 + 64)
    m, o = baseline_pair(cfg, seed=2)
    kw = dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1, repetition_context=256, seed=3)
    prompt = cuda.synth_prompt(8192, cfg.vocab, seed=2)
    kv = m.new_kv(4096 + 512 - 1)
    gt, glp, _ = m.generate(prompt, 48, sp=cuda.sampling(**kw), logprobs=True, kv=kv, chunk=512)
    ot, olp, _ = o.generate(prompt, 48, sp=po.sampling(**kw), chunk=512)
    assert len(gt) == 48
    assert np.array_equal(gt, ot)
    assert np.abs(glp - olp).max() < 1e-4


def test_config_c5_llama3_70b_shortened():
    """C5 shortened to 2 layers on one GPU: Llama-3-70B width (hidden 8192,
    64/8 heads, head dim 128, MLP 28672, vocab 128256) with the llama3-scaled
    RoPE (theta 500000, factor 8, low 1, high 4, original 8192), 512 prompt
    ids then 32 greedy tokens: identical tokens and first-position logits."""
    cfg = cuda.synth_config(hidden=8192, layers=2, n_heads=64, n_kv_heads=8, head_dim=128, inter=28672,
                            vocab=128256, family=cuda.LLAMA, theta=500000.0, llama3=(8.0, 1.0, 4.0, 8192),
                            max_pos=1024)
    gt, ot, g, ol, (ok, mx, mr) = run_config(cfg, 512, 32)
    assert np.array_equal(gt, ot) and len(gt) == 32
    assert same_bits(g, ol) and ok
