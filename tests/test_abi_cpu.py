"""CPU-side checks of the C ABI library: it loads without a GPU, exports every
symbol include/mlxd_cuda.h declares, and its host-side synthetic generator
matches the oracle's restatement of mlx affine quantisation."""
import os
import re

import numpy as np
import pytest

from mlxd_b200 import cuda
from oracle import pyoracle as po
from tests.helpers import bf16_to_f32

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "mlxd_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mlxd_(?:cuda|host)_\w+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    L = cuda.lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(syms) == set(cuda._SIGS), set(syms) ^ set(cuda._SIGS)


def test_engine_library_exports_every_declared_function():
    """libmlxd_engine (the C11 engine surface) exports every function its
    header mlxd_engine.h declares."""
    import ctypes
    lib = os.path.join(ROOT, "mlxd_b200", "libmlxd_engine.so")
    if not os.path.exists(lib):
        pytest.skip("libmlxd_engine.so not built")
    L = ctypes.CDLL(lib)
    src = open(os.path.join(ROOT, "mlxd_b200", "engine", "mlxd_engine.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"#define[^\n]*(\\\n[^\n]*)*", "", src)
    names = sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", src)))
    for want in ("engine_model_load", "model_forward", "kvcache_update", "sampler_sample_lazy",
                 "mlxbridge_async_eval_n", "mlxbridge_item_int32", "mlx_reshape", "mlxd_checkpoint_open"):
        assert want in names
    assert len(names) >= 35, names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_last_error_is_empty_string_initially():
    assert cuda.lib().mlxd_cuda_last_error() == b""


def test_host_synth_deterministic_and_normal():
    a = np.zeros(1 << 16, np.uint16)
    b = np.zeros(1 << 16, np.uint16)
    L = cuda.lib()
    L.mlxd_host_synth_bf16(cuda.ptr(a), a.size, 7, 0.02, 0.0)
    L.mlxd_host_synth_bf16(cuda.ptr(b), b.size, 7, 0.02, 0.0)
    assert np.array_equal(a, b)
    v = bf16_to_f32(a)
    assert abs(v.mean()) < 1e-3 and abs(v.std() - 0.02) < 1e-3
    L.mlxd_host_synth_bf16(cuda.ptr(b), b.size, 8, 0.02, 0.0)
    assert not np.array_equal(a, b)


@pytest.mark.parametrize("group", [64, 32])
def test_host_quantizer_matches_oracle_restatement(group):
    rows, cols = 48, 256
    w = np.zeros((rows, cols // 8), np.uint32)
    s = np.zeros((rows, cols // group), np.uint16)
    b = np.zeros((rows, cols // group), np.uint16)
    cuda.lib().mlxd_host_synth_quantized(cuda.ptr(w), cuda.ptr(s), cuda.ptr(b), rows, cols,
                                         group, 11, 0.02)
    # the same N(0, 0.02) bf16 values, quantised by the oracle
    vals = np.zeros(rows * cols, np.uint16)
    cuda.lib().mlxd_host_synth_bf16(cuda.ptr(vals), vals.size, 11, 0.02, 0.0)
    wf = bf16_to_f32(vals).reshape(rows, cols)
    wq, so, bo = po.affine_quantize(wf, group)
    assert np.array_equal(wq, w)
    assert np.array_equal(po.f32_to_bf16(so), s)
    assert np.array_equal(po.f32_to_bf16(bo), b)
    # dequantisation error within one level (mlx's edge-snapped scale can clip
    # the opposite extreme by up to one level), plus the bf16 rounding of the
    # stored scale (over 15 levels) and bias
    sc = bf16_to_f32(s).repeat(group, axis=1)
    bi = bf16_to_f32(b).repeat(group, axis=1)
    q = np.stack([(w >> (4 * k)) & 0xF for k in range(8)], axis=-1).reshape(rows, cols)
    deq = sc * q + bi
    bound = np.abs(sc) * (1.0 + 15 * 2.0 ** -8) + np.abs(bi) * 2.0 ** -8 + 1e-6
    assert np.all(np.abs(deq - wf) <= bound)


def test_config_from_fixture(golden_dir):
    import json
    for name in ("tiny_qwen3", "tiny_qwen3_tied", "tiny_qwen3_5_tied", "tiny_llama3",
                 "tiny_mistral"):
        cj = json.load(open(os.path.join(golden_dir, name, "config.json")))
        c = cuda.config_from_json(cj)
        assert c.hidden == 64 and c.head_dim == 16 and c.layers == 2
        if name == "tiny_qwen3_5_tied":
            assert c.attn_gate == 1 and c.rope_dims == 4 and c.qbits == 4 and c.qgroup == 32
        if name == "tiny_mistral":
            assert c.window == 8
        if name == "tiny_llama3":
            assert c.rope_llama3 == 1 and c.rope_orig_max == 8192


def test_qwen3_rejects_rope_scaling():
    cj = {"model_type": "qwen3", "vocab_size": 8, "hidden_size": 16, "num_hidden_layers": 1,
          "num_attention_heads": 1, "rope_scaling": {"rope_type": "linear", "factor": 2.0}}
    with pytest.raises(ValueError):
        cuda.config_from_json(cj)


def test_synth_prompt_uniform():
    p = cuda.synth_prompt(20000, 151936, seed=3)
    assert p.min() >= 0 and p.max() < 151936
    assert np.array_equal(p, cuda.synth_prompt(20000, 151936, seed=3))
    assert abs(p.mean() / 151936 - 0.5) < 0.02


def test_oracle_synth_matches_library_synth():
    """The CPU baseline builds its weights with the oracle's copy of the
    generator (no CUDA library in that process): same bits as the library's."""
    cfg = cuda.synth_config(hidden=128, layers=1, n_heads=2, n_kv_heads=1, head_dim=64, inter=256,
                            vocab=512)
    specs = cuda.synth_tensor_specs(cfg)
    a = cuda.synth_host_tensors(cfg, seed=5)
    b = po.synth_host_tensors(specs, cfg.qgroup, seed=5)
    assert a.keys() == b.keys()
    for k in a:
        assert np.array_equal(a[k], b[k]), k
    L = cuda.lib()
    for group in (32, 64):
        w = np.zeros((48, 320 // 8), np.uint32)
        s = np.zeros((48, 320 // group), np.uint16)
        bb = np.zeros_like(s)
        L.mlxd_host_synth_quantized(cuda.ptr(w), cuda.ptr(s), cuda.ptr(bb), 48, 320, group, 99, 0.06)
        w2, s2, b2 = np.zeros_like(w), np.zeros_like(s), np.zeros_like(bb)
        po.lib().orc_synth_quantized(po.ptr(w2), po.ptr(s2), po.ptr(b2), 48, 320, group, 99, 0.06)
        assert np.array_equal(w, w2) and np.array_equal(s, s2) and np.array_equal(bb, b2)
