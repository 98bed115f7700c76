"""The C11 engine surface (libmlxd_engine, mlxd_engine.h) driven by a compiled
C program (tests/c/test_engine.c) in the reference's own generate pattern:
model directory loaded by the C loader, chunked prefill and seed forward
through model_forward, the pipelined decode through sampler_sample_lazy,
mlx_reshape, mlxbridge_async_eval_n and mlxbridge_item_int32. Tokens are
checked against the oracle (greedy) and against mlxd_cuda_generate (seeded
sampling, same draw stream); the async pair and the KV views too."""
import os
import subprocess

import numpy as np
import pytest

from mlxd_b200 import cuda
from oracle import pyoracle as po

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
PKG = os.path.join(ROOT, "mlxd_b200")


@pytest.fixture(scope="module")
def prog(tmp_path_factory):
    if not os.path.exists(os.path.join(PKG, "libmlxd_engine.so")):
        subprocess.check_call(["make", "-C", os.path.join(PKG, "engine")])
    out = str(tmp_path_factory.mktemp("c") / "test_engine")
    subprocess.check_call(["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I" + os.path.join(ROOT, "include"),
                           "-I" + os.path.join(PKG, "engine"), os.path.join(HERE, "c", "test_engine.c"), "-o", out,
                           "-L" + PKG, "-l:libmlxd_engine.so", "-l:libmlxd_cuda.so", "-Wl,-rpath," + PKG])
    return out


def run(prog, *args):
    r = subprocess.run([prog] + [str(a) for a in args], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    out = {}
    for line in r.stdout.splitlines():
        k, _, v = line.partition(" ")
        out[k] = v.split()
    return out


FIXTURES = ["tiny_qwen3", "tiny_qwen3_5_tied", "tiny_llama3", "tiny_mistral_tied"]
PROMPT = [3, 17, 91, 4, 55, 200, 8, 1, 13, 77, 42, 9]


@pytest.mark.parametrize("name", FIXTURES)
def test_c_generate_greedy_matches_oracle(prog, name):
    d = os.path.join(GOLDEN, name)
    out = run(prog, "generate", d, 16, 5, 0.0, -1, 1.0, -1, *PROMPT)
    toks = [int(t) for t in out["TOKENS"]]
    o = po.Oracle.from_dir(d)
    ot, olp, _ = o.generate(PROMPT, 16, chunk=5)
    assert toks == list(map(int, ot))
    assert np.abs(np.array([float(x) for x in out["LOGPROBS"]]) - olp).max() < 1e-4
    assert int(out["OFFSET"][0]) == len(PROMPT) + len(toks) - 1


def test_c_kOracle_ids(prog, goldens):
    g = goldens["kOracle"]
    out = run(prog, "generate", os.path.join(GOLDEN, g["fixture"]), g["max_tokens"], 512, 0.0, -1, 1.0, -1,
              *g["prompt"])
    assert [int(t) for t in out["TOKENS"]] == g["ids"]


@pytest.mark.parametrize("name", ["tiny_qwen3", "tiny_mistral_tied"])
def test_c_generate_seeded_sampling_matches_library_generate(prog, name):
    d = os.path.join(GOLDEN, name)
    out = run(prog, "generate", d, 20, 512, 0.8, 40, 0.9, 11, *PROMPT)
    cuda.init(0)
    m = cuda.Model.from_dir(d)
    gt, glp, _ = m.generate(PROMPT, 20, sp=cuda.sampling(temperature=0.8, top_k=40, top_p=0.9, seed=11),
                            logprobs=True)
    m.close()
    assert [int(t) for t in out["TOKENS"]] == list(map(int, gt))
    assert np.abs(np.array([float(x) for x in out["LOGPROBS"]]) - glp).max() < 1e-6


@pytest.mark.parametrize("name", ["tiny_qwen3", "tiny_qwen3_5_tied"])
def test_c_async_pair_matches_oracle(prog, name):
    d = os.path.join(GOLDEN, name)
    out = run(prog, "async", d, 12, *PROMPT)
    ot, _, _ = po.Oracle.from_dir(d).generate(PROMPT, 12)
    assert [int(t) for t in out["TOKENS"]][:len(ot)] == list(map(int, ot))


@pytest.mark.parametrize("name", ["tiny_qwen3", "tiny_mistral_tied"])
def test_c_kvcache_views(prog, name):
    out = run(prog, "kv", os.path.join(GOLDEN, name), *PROMPT)
    assert "KV" in out


def test_c_load_reports_validation_errors(prog, tmp_path):
    d = str(tmp_path / "m")
    os.makedirs(d)
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write('{"model_type": "gemma3", "vocab_size": 8, "hidden_size": 8, "num_hidden_layers": 1,'
                ' "num_attention_heads": 1}')
    out = run(prog, "load", d)
    assert out["LOAD"][0] == "ERROR" and "unsupported model family" in " ".join(out["LOAD"])
    out = run(prog, "load", os.path.join(GOLDEN, "tiny_qwen3"))
    assert out["LOAD"] == ["OK"]
