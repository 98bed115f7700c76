"""The C11 model-directory loader of libmlxd_engine on the CPU (no GPU call):
config.json parsing against the Python reader, the support gate, shard
enumeration and the reference's weight validation
(src/model/weights.c:20-192, 651-940; src/engine/emodel.c:22-150), each
failure with the reference's message."""
import ctypes as C
import json
import os
import struct

import numpy as np
import pytest

from mlxd_b200 import cuda

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
LIB = os.path.join(ROOT, "mlxd_b200", "libmlxd_engine.so")


class ModelConfigT(C.Structure):
    """model_config_t of mlxd_engine.h"""
    _fields_ = [("model_type", C.c_char * 32),
                ("vocab_size", C.c_int), ("hidden_size", C.c_int), ("num_hidden_layers", C.c_int),
                ("num_attention_heads", C.c_int), ("num_key_value_heads", C.c_int),
                ("max_position_embeddings", C.c_int), ("intermediate_size", C.c_int), ("head_dim", C.c_int),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
                ("rope_scaling_type", C.c_char * 16),
                ("rope_scaling_factor", C.c_float), ("rope_low_freq_factor", C.c_float),
                ("rope_high_freq_factor", C.c_float), ("rope_original_max_position_embeddings", C.c_int),
                ("partial_rotary_factor", C.c_float),
                ("has_sliding_window", C.c_bool), ("sliding_window", C.c_int), ("attention_bias", C.c_bool),
                ("quant_bits", C.c_int), ("quant_group_size", C.c_int),
                ("tie_word_embeddings", C.c_bool), ("has_qk_norm", C.c_bool), ("attn_output_gate", C.c_bool),
                ("hidden_act_silu", C.c_bool), ("num_experts", C.c_int),
                ("num_eos_tokens", C.c_int), ("eos_token_ids", C.c_int * 8),
                ("has_gen_temperature", C.c_bool), ("has_gen_top_p", C.c_bool), ("has_gen_top_k", C.c_bool),
                ("gen_temperature", C.c_float), ("gen_top_p", C.c_float), ("gen_top_k", C.c_int)]


class Checkpoint(C.Structure):
    _fields_ = [("tensors", C.POINTER(cuda.Tensor)), ("n_tensors", C.c_int), ("maps", C.c_void_p),
                ("map_sizes", C.c_void_p), ("n_maps", C.c_int)]


@pytest.fixture(scope="module")
def eng():
    if not os.path.exists(LIB):
        pytest.skip("libmlxd_engine.so not built")
    L = C.CDLL(LIB)
    L.model_config_load.argtypes = [C.POINTER(ModelConfigT), C.c_char_p, C.c_char_p, C.c_size_t]
    L.model_config_to_cuda.argtypes = [C.POINTER(ModelConfigT), C.c_int, C.c_int, C.POINTER(cuda.ModelConfig),
                                       C.c_char_p, C.c_size_t]
    L.engine_model_check_supported.argtypes = [C.POINTER(ModelConfigT), C.c_char_p, C.c_size_t]
    L.mlxd_checkpoint_open.argtypes = [C.POINTER(Checkpoint), C.c_char_p, C.POINTER(ModelConfigT), C.c_char_p,
                                       C.c_size_t]
    L.mlxd_checkpoint_close.argtypes = [C.POINTER(Checkpoint)]
    return L


def load_cfg(L, d):
    c = ModelConfigT()
    err = C.create_string_buffer(512)
    rc = L.model_config_load(C.byref(c), d.encode(), err, 512)
    return rc, c, err.value.decode()


def open_ck(L, d):
    rc, c, err = load_cfg(L, d)
    assert rc == 0, err
    ck = Checkpoint()
    e = C.create_string_buffer(512)
    rc = L.mlxd_checkpoint_open(C.byref(ck), d.encode(), C.byref(c), e, 512)
    return rc, ck, e.value.decode()


FIXTURES = ["tiny_qwen3", "tiny_qwen3_tied", "tiny_qwen3_5", "tiny_qwen3_5_tied", "tiny_llama3",
            "tiny_llama3_tied", "tiny_mistral", "tiny_mistral_tied"]


@pytest.mark.parametrize("name", FIXTURES)
def test_config_matches_python_reader(eng, name):
    d = os.path.join(GOLDEN, name)
    rc, c, err = load_cfg(eng, d)
    assert rc == 0, err
    mc = cuda.ModelConfig()
    e = C.create_string_buffer(512)
    assert eng.model_config_to_cuda(C.byref(c), 0, 1, C.byref(mc), e, 512) == 0, e.value
    py = cuda.config_from_json(json.load(open(os.path.join(d, "config.json"))))
    for f, _ in cuda.ModelConfig._fields_:
        a, b = getattr(mc, f), getattr(py, f)
        if hasattr(a, "__len__"):
            assert list(a) == list(b), f
        elif isinstance(a, float):
            assert a == pytest.approx(b, rel=1e-7), f
        else:
            assert a == b, f


@pytest.mark.parametrize("name", FIXTURES)
def test_checkpoint_lists_every_tensor(eng, name):
    d = os.path.join(GOLDEN, name)
    rc, ck, err = open_ck(eng, d)
    assert rc == 0, err
    want = cuda.read_checkpoint(d)
    got = {}
    for i in range(ck.n_tensors):
        t = ck.tensors[i]
        shape = tuple(t.shape[:t.ndim])
        nbytes = int(np.prod(shape)) * (2 if t.dtype == cuda.BF16 else 4)
        got[t.name.decode()] = (shape, C.string_at(t.data, nbytes))
    assert set(got) == set(want)
    for k, a in want.items():
        assert got[k][0] == a.shape and got[k][1] == a.tobytes(), k
    eng.mlxd_checkpoint_close(C.byref(ck))


# ------------------------------------------------ synthetic directories

def write_st(path, tensors):
    """safetensors writer: {name: ndarray}"""
    hdr, blobs, off = {}, [], 0
    dt = {np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32",
          np.dtype(np.float16): "F16"}
    for k, a in tensors.items():
        b = a.tobytes()
        hdr[k] = {"dtype": dt[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def tiny_model(d, quant=True, **cfg_over):
    cfg = dict(model_type="qwen3", vocab_size=64, hidden_size=64, num_hidden_layers=2, num_attention_heads=2,
               num_key_value_heads=1, head_dim=32, intermediate_size=64, max_position_embeddings=128,
               rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True)
    if quant:
        cfg["quantization"] = {"bits": 4, "group_size": 64}
    cfg.update(cfg_over)
    os.makedirs(d, exist_ok=True)
    json.dump(cfg, open(os.path.join(d, "config.json"), "w"))
    H = cfg["hidden_size"]
    t = {}

    def proj(name, rows, cols):
        if quant:
            t[name + ".weight"] = np.zeros((rows, cols // 8), np.uint32)
            t[name + ".scales"] = np.ones((rows, cols // 64), np.uint16)
            t[name + ".biases"] = np.zeros((rows, cols // 64), np.uint16)
        else:
            t[name + ".weight"] = np.zeros((rows, cols), np.uint16)

    proj("model.embed_tokens", cfg["vocab_size"], H)
    t["model.norm.weight"] = np.ones(H, np.uint16)
    for l in range(cfg["num_hidden_layers"]):
        p = "model.layers.%d." % l
        qd, kd = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]
        for n, r, c in (("self_attn.q_proj", qd, H), ("self_attn.k_proj", kd, H), ("self_attn.v_proj", kd, H),
                        ("self_attn.o_proj", H, qd), ("mlp.gate_proj", cfg["intermediate_size"], H),
                        ("mlp.up_proj", cfg["intermediate_size"], H), ("mlp.down_proj", H, cfg["intermediate_size"])):
            proj(p + n, r, c)
        for n in ("input_layernorm", "post_attention_layernorm", "self_attn.q_norm", "self_attn.k_norm"):
            t[p + n + ".weight"] = np.ones(cfg["head_dim"] if "norm." in n + "." and "self_attn" in n else H,
                                           np.uint16)
    return t


def shard(d, t, parts):
    """split tensors over `parts` files with an index"""
    names = sorted(t)
    wm = {}
    for i in range(parts):
        fn = "model-%05d-of-%05d.safetensors" % (i + 1, parts)
        sub = {k: t[k] for k in names[i::parts]}
        write_st(os.path.join(d, fn), sub)
        wm.update({k: fn for k in sub})
    json.dump({"weight_map": wm}, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    return wm


def test_synthetic_single_file_and_shards_load(eng, tmp_path):
    d = str(tmp_path / "one")
    t = tiny_model(d)
    write_st(os.path.join(d, "model.safetensors"), t)
    rc, ck, err = open_ck(eng, d)
    assert rc == 0, err
    assert ck.n_tensors == len(t)
    eng.mlxd_checkpoint_close(C.byref(ck))
    d2 = str(tmp_path / "three")
    t = tiny_model(d2)
    shard(d2, t, 3)
    rc, ck, err = open_ck(eng, d2)
    assert rc == 0, err
    assert ck.n_tensors == len(t)
    eng.mlxd_checkpoint_close(C.byref(ck))


def expect_error(eng, d, text):
    rc, ck, err = open_ck(eng, d)
    assert rc != 0 and text in err, err


def test_duplicate_tensor_across_shards(eng, tmp_path):
    d = str(tmp_path / "m")
    t = tiny_model(d)
    shard(d, t, 2)
    # the norm also in a third shard the index names
    write_st(os.path.join(d, "model-extra.safetensors"), {"model.norm.weight": t["model.norm.weight"]})
    idx = json.load(open(os.path.join(d, "model.safetensors.index.json")))
    idx["weight_map"]["model.norm.weight"] = "model-extra.safetensors"
    json.dump(idx, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    expect_error(eng, d, 'duplicate tensor "model.norm.weight"')


def test_index_declares_missing_tensor(eng, tmp_path):
    d = str(tmp_path / "m")
    t = tiny_model(d)
    shard(d, t, 2)
    idx = json.load(open(os.path.join(d, "model.safetensors.index.json")))
    idx["weight_map"]["model.layers.0.extra.weight"] = "model-00001-of-00002.safetensors"
    json.dump(idx, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    expect_error(eng, d, 'index declares tensor "model.layers.0.extra.weight" but it was not found')


def test_index_with_path_in_file_name_is_invalid(eng, tmp_path):
    d = str(tmp_path / "m")
    t = tiny_model(d)
    shard(d, t, 2)
    idx = json.load(open(os.path.join(d, "model.safetensors.index.json")))
    k = next(iter(idx["weight_map"]))
    idx["weight_map"][k] = "../evil.safetensors"
    json.dump(idx, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    expect_error(eng, d, "invalid model.safetensors.index.json")


def test_missing_layer_and_expected_tensor(eng, tmp_path):
    d = str(tmp_path / "a")
    t = tiny_model(d)
    for k in [k for k in t if k.startswith("model.layers.1.")]:
        del t[k]
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, "missing tensors for layer 1")
    d = str(tmp_path / "b")
    t = tiny_model(d)
    del t["model.layers.0.self_attn.k_norm.weight"]
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'missing expected tensor "model.layers.0.self_attn.k_norm.weight"')
    d = str(tmp_path / "c")
    t = tiny_model(d, tie_word_embeddings=False)
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'missing expected tensor "lm_head.weight"')


def test_orphan_scales_and_biases(eng, tmp_path):
    d = str(tmp_path / "a")
    t = tiny_model(d)
    t["model.layers.0.mlp.extra.scales"] = np.ones((4, 1), np.uint16)
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'orphan .scales for "model.layers.0.mlp.extra" (base .weight missing)')
    d = str(tmp_path / "b")
    t = tiny_model(d)
    del t["model.layers.1.mlp.up_proj.biases"]
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'orphan .scales for "model.layers.1.mlp.up_proj" (missing .biases)')


def test_quantized_dtypes(eng, tmp_path):
    d = str(tmp_path / "a")
    t = tiny_model(d)
    w = t["model.layers.0.self_attn.q_proj.weight"]
    t["model.layers.0.self_attn.q_proj.weight"] = np.zeros((w.shape[0], w.shape[1] * 2), np.uint16)
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, "quantized weight model.layers.0.self_attn.q_proj.weight has dtype")
    d = str(tmp_path / "b")
    t = tiny_model(d, quant=False)
    t["model.layers.0.self_attn.q_proj.weight"] = np.zeros((64, 8), np.uint32)
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'is uint32 but config has no quantization')
    d = str(tmp_path / "c")
    t = tiny_model(d)
    t["model.norm.weight"] = np.ones(64, np.float16)
    write_st(os.path.join(d, "model.safetensors"), t)
    expect_error(eng, d, 'unsupported dtype F16')
    d = str(tmp_path / "e")
    os.makedirs(d)
    json.dump({"model_type": "qwen3", "vocab_size": 8, "hidden_size": 8, "num_hidden_layers": 1,
               "num_attention_heads": 1}, open(os.path.join(d, "config.json"), "w"))
    expect_error(eng, d, "no safetensors files found")


@pytest.mark.parametrize("over,text", [
    (dict(rope_scaling={"rope_type": "llama3", "factor": 8.0}), "RoPE scaling not supported"),
    (dict(attention_bias=True), "attention_bias not supported"),
    (dict(num_experts=8), "MoE models not supported"),
    (dict(hidden_act="gelu"), "only SiLU activation supported"),
    (dict(model_type="gemma3"), "unsupported model family"),
    (dict(model_type="llama", rope_scaling={"rope_type": "yarn"}), "unsupported RoPE scaling type"),
    (dict(model_type="qwen3_5", attn_output_gate=False), "qwen3_5 requires attn_output_gate"),
    (dict(model_type="qwen3_5", partial_rotary_factor=0.1), "invalid rope dims"),
])
def test_support_gate(eng, tmp_path, over, text):
    d = str(tmp_path / "m")
    tiny_model(d, **over)
    rc, c, err = load_cfg(eng, d)
    assert rc == 0, err
    e = C.create_string_buffer(512)
    assert eng.engine_model_check_supported(C.byref(c), e, 512) != 0
    assert text in e.value.decode(), e.value


def test_generation_config_defaults(eng, tmp_path):
    d = str(tmp_path / "m")
    tiny_model(d)
    json.dump({"temperature": 0.6, "top_p": 0.95, "top_k": 20, "eos_token_id": [5, 7]},
              open(os.path.join(d, "generation_config.json"), "w"))
    rc, c, err = load_cfg(eng, d)
    assert rc == 0, err
    assert c.has_gen_temperature and c.gen_temperature == pytest.approx(0.6)
    assert c.has_gen_top_p and c.gen_top_p == pytest.approx(0.95)
    assert c.has_gen_top_k and c.gen_top_k == 20
    assert c.num_eos_tokens == 2 and list(c.eos_token_ids[:2]) == [5, 7]
