"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. It loads oracle/liboracle.so (built by oracle/Makefile), reads
MLX-format checkpoints (config.json + safetensors) with numpy, and restates
the reference's config defaults (src/model/model.c:160-175, 350-385, 667-1031)
for the dense families on the path (qwen3, llama, mistral, qwen3_5).
"""
import ctypes as C
import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

QWEN3, LLAMA, MISTRAL, QWEN3_5 = 1, 2, 3, 4
BF16, F32, U32 = 1, 2, 3
_DT = {"BF16": (BF16, np.uint16), "F32": (F32, np.float32), "U32": (U32, np.uint32)}


class OrcConfig(C.Structure):
    _fields_ = [("family", C.c_int), ("vocab", C.c_int), ("hidden", C.c_int),
                ("layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("max_pos", C.c_int),
                ("eps", C.c_float), ("rope_theta", C.c_float), ("qk_norm", C.c_int),
                ("tie", C.c_int), ("attn_gate", C.c_int), ("rope_dims", C.c_int),
                ("rope_llama3", C.c_int), ("rope_factor", C.c_float),
                ("rope_lo", C.c_float), ("rope_hi", C.c_float), ("rope_orig_max", C.c_int),
                ("window", C.c_int), ("qbits", C.c_int), ("qgroup", C.c_int),
                ("n_eos", C.c_int), ("eos", C.c_int * 8)]


class OrcSampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("min_p", C.c_float), ("seed", C.c_int),
                ("repetition_penalty", C.c_float), ("repetition_context", C.c_int)]


def sampling(temperature=1.0, top_p=1.0, top_k=-1, min_p=0.0, seed=-1,
             repetition_penalty=1.0, repetition_context=20):
    """SAMPLING_PARAMS_DEFAULT (src/core/types.h:34-35) plus the build-defined
    repetition penalty (off at 1.0)."""
    return OrcSampling(temperature, top_p, top_k, min_p, seed,
                       repetition_penalty, repetition_context)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("oracle not built: run make -C oracle")
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        L.orc_model_new.restype = P
        L.orc_model_new.argtypes = [C.POINTER(OrcConfig)]
        L.orc_model_set_tensor.argtypes = [P, C.c_char_p, C.c_int, C.POINTER(C.c_int64), C.c_int, P]
        L.orc_model_finalize.argtypes = [P, C.c_char_p, C.c_int]
        L.orc_model_free.argtypes = [P]
        L.orc_kv_new.restype = P
        L.orc_kv_new.argtypes = [P, C.c_int]
        L.orc_kv_free.argtypes = [P]
        L.orc_kv_offset.argtypes = [P, C.c_int]
        L.orc_kv_read.argtypes = [P, C.c_int, C.c_int, P]
        L.orc_forward.argtypes = [P, P, P, C.c_int, C.c_int, P]
        L.orc_synth_quantized.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_float]
        L.orc_synth_bf16.argtypes = [P, C.c_size_t, C.c_uint64, C.c_float, C.c_float]
        L.orc_synth_bf16.restype = None
        L.orc_kv_fill_synth.argtypes = [P, C.c_int, C.c_uint64]
        L.orc_forward_hidden.argtypes = [P, P, P, C.c_int, P]
        L.orc_qlinear.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P, P, C.c_int, C.c_int, C.c_int, P]
        L.orc_dense_linear.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P]
        L.orc_rmsnorm.argtypes = [P, C.c_int, C.c_int, P, C.c_float, P]
        L.orc_rope.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_float, P]
        L.orc_rope_llama3_freqs.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float,
                                            C.c_int, C.c_int, P]
        L.orc_affine_quantize.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P, P]
        L.orc_sample.argtypes = [P, C.c_int, C.POINTER(OrcSampling), P, C.c_int, C.c_uint64,
                                 P, P, P]
        L.orc_top_k.argtypes = [P, C.c_int, C.c_int]
        L.orc_top_p.argtypes = [P, C.c_int, C.c_float]
        L.orc_min_p.argtypes = [P, C.c_int, C.c_float]
        L.orc_expf.argtypes = [C.c_float]
        L.orc_expf.restype = C.c_float
        L.orc_generate.argtypes = [P, P, C.c_int, C.c_int, C.POINTER(OrcSampling), C.c_int,
                                   P, P, P]
        L.orc_window_mask.argtypes = [C.c_int, C.c_int, C.c_int, P]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _lib = L
    return _lib


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------- files

def read_safetensors(path):
    """8-byte LE header length, JSON header, raw little-endian tensors."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, meta in hdr.items():
            if name == "__metadata__":
                continue
            code, npdt = _DT[meta["dtype"]]
            a, b = meta["data_offsets"]
            f.seek(base + a)
            arr = np.frombuffer(f.read(b - a), dtype=npdt).reshape(meta["shape"]).copy()
            out[name] = arr
        return out


def read_checkpoint(model_dir):
    idx = os.path.join(model_dir, "model.safetensors.index.json")
    tensors = {}
    if os.path.exists(idx):
        files = sorted(set(json.load(open(idx))["weight_map"].values()))
    else:
        files = ["model.safetensors"]
    for fn in files:
        tensors.update(read_safetensors(os.path.join(model_dir, fn)))
    return tensors


def config_from_json(cj):
    """model_config_load (model.c:667-1031) defaults for the dense families."""
    fam = {"qwen3": QWEN3, "llama": LLAMA, "mistral": MISTRAL,
           "qwen3_5": QWEN3_5, "qwen3_5_text": QWEN3_5}[cj["model_type"]]
    c = OrcConfig()
    c.family = fam
    c.vocab = cj["vocab_size"]
    c.hidden = cj["hidden_size"]
    c.layers = cj["num_hidden_layers"]
    c.n_heads = cj["num_attention_heads"]
    c.n_kv_heads = cj.get("num_key_value_heads", c.n_heads)
    c.head_dim = cj.get("head_dim") or c.hidden // c.n_heads
    c.inter = cj.get("intermediate_size", 0)
    c.max_pos = cj.get("max_position_embeddings", 0)
    c.eps = cj.get("rms_norm_eps", 1e-6)
    theta = cj.get("rope_theta", 1e6)
    prf = 1.0
    rp = cj.get("rope_parameters")
    if isinstance(rp, dict) and not any(isinstance(v, dict) for v in rp.values()):
        theta = rp.get("rope_theta", theta)
        prf = rp.get("partial_rotary_factor", prf)
    c.rope_theta = theta
    c.qk_norm = 1 if fam in (QWEN3, QWEN3_5) else 0
    c.tie = 1 if cj.get("tie_word_embeddings", False) else 0
    c.attn_gate = 1 if (fam == QWEN3_5 and cj.get("attn_output_gate", True)) else 0
    c.rope_dims = int(c.head_dim * prf) if prf != 1.0 else c.head_dim
    rs = cj.get("rope_scaling")
    if isinstance(rs, dict) and (rs.get("rope_type") or rs.get("type")) == "llama3":
        c.rope_llama3 = 1
        c.rope_factor = rs.get("factor", 1.0)
        c.rope_lo = rs.get("low_freq_factor", 1.0)
        c.rope_hi = rs.get("high_freq_factor", 1.0)
        c.rope_orig_max = rs.get("original_max_position_embeddings", 0)
    sw = cj.get("sliding_window")
    c.window = int(sw) if (fam == MISTRAL and isinstance(sw, int) and sw > 0) else 0
    q = cj.get("quantization")
    c.qbits = q["bits"] if q else 0
    c.qgroup = q.get("group_size", 64) if q else 64
    eos = cj.get("eos_token_id")
    eos = [] if eos is None else (eos if isinstance(eos, list) else [eos])
    c.n_eos = len(eos)
    for i, e in enumerate(eos[:8]):
        c.eos[i] = e
    return c


# ----------------------------------------------------------------- model

class Oracle:
    def __init__(self, cfg, tensors):
        L = lib()
        self.cfg = cfg
        self.m = L.orc_model_new(C.byref(cfg))
        for name, arr in tensors.items():
            arr = np.ascontiguousarray(arr)
            code = {np.uint16: BF16, np.float32: F32, np.uint32: U32}[arr.dtype.type]
            shape = (C.c_int64 * arr.ndim)(*arr.shape)
            if L.orc_model_set_tensor(self.m, name.encode(), code, shape, arr.ndim, ptr(arr)):
                raise RuntimeError("set_tensor failed: " + name)
        err = C.create_string_buffer(256)
        if L.orc_model_finalize(self.m, err, 256):
            raise RuntimeError("oracle finalize: " + err.value.decode())

    @classmethod
    def from_dir(cls, model_dir):
        cj = json.load(open(os.path.join(model_dir, "config.json")))
        return cls(config_from_json(cj), read_checkpoint(model_dir))

    def __del__(self):
        if getattr(self, "m", None):
            lib().orc_model_free(self.m)
            self.m = None

    def new_kv(self, capacity):
        return KV(self, capacity)

    def forward(self, kv, ids, want_logits=True):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(self.cfg.vocab, dtype=np.float32)
        rc = lib().orc_forward(self.m, kv.kv, ptr(ids), len(ids), int(want_logits), ptr(out))
        if rc:
            raise RuntimeError("oracle forward failed")
        return out if want_logits else None

    def forward_hidden(self, kv, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((len(ids), self.cfg.hidden), dtype=np.uint16)
        if lib().orc_forward_hidden(self.m, kv.kv, ptr(ids), len(ids), ptr(out)):
            raise RuntimeError("oracle forward failed")
        return out

    def generate(self, prompt, max_new, sp=None, chunk=512):
        sp = sp or sampling(temperature=0.0)
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_new, dtype=np.int32)
        lps = np.zeros(max_new, dtype=np.float32)
        margins = np.zeros(max_new, dtype=np.float32)
        n = lib().orc_generate(self.m, ptr(prompt), len(prompt), max_new, C.byref(sp), chunk,
                               ptr(out), ptr(lps), ptr(margins))
        if n < 0:
            raise RuntimeError("oracle generate failed (%d)" % n)
        return out[:n], lps[:n], margins[:n]


class KV:
    def __init__(self, orc, capacity):
        self.orc = orc
        self.kv = lib().orc_kv_new(orc.m, capacity)

    def offset(self, layer=0):
        return lib().orc_kv_offset(self.kv, layer)

    def read(self, layer, value=False):
        c = self.orc.cfg
        off = self.offset(layer)
        out = np.zeros((c.n_kv_heads, off, c.head_dim), dtype=np.uint16)
        lib().orc_kv_read(self.kv, layer, int(value), ptr(out))
        return out

    def __del__(self):
        if getattr(self, "kv", None):
            lib().orc_kv_free(self.kv)
            self.kv = None


# ----------------------------------------------------------------- ops

def bf16_to_f32(a):
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def qlinear(x_bf16, w, scales, biases, group, exact=True):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    S = 1 if x.ndim == 1 else x.shape[0]
    out_f, in_f = w.shape[0], w.shape[1] * 8
    sdt = F32 if scales.dtype == np.float32 else BF16
    y = np.zeros((S, out_f), dtype=np.uint16)
    lib().orc_qlinear(ptr(x), S, in_f, out_f, ptr(np.ascontiguousarray(w)),
                      ptr(np.ascontiguousarray(scales)), ptr(np.ascontiguousarray(biases)),
                      sdt, group, int(exact), ptr(y))
    return y


def dense_linear(x_bf16, w_bf16):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    S = 1 if x.ndim == 1 else x.shape[0]
    y = np.zeros((S, w_bf16.shape[0]), dtype=np.uint16)
    lib().orc_dense_linear(ptr(x), S, w_bf16.shape[1], w_bf16.shape[0],
                           ptr(np.ascontiguousarray(w_bf16)), ptr(y))
    return y


def rmsnorm(x_bf16, w_bf16, eps):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    n = x.shape[-1]
    rows = x.size // n
    y = np.zeros_like(x)
    lib().orc_rmsnorm(ptr(x), rows, n, ptr(np.ascontiguousarray(w_bf16)), eps, ptr(y))
    return y


def affine_quantize(w_f32, group):
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    rows, cols = w.shape
    wq = np.zeros((rows, cols // 8), dtype=np.uint32)
    s = np.zeros((rows, cols // group), dtype=np.float32)
    b = np.zeros((rows, cols // group), dtype=np.float32)
    lib().orc_affine_quantize(ptr(w), rows, cols, group, ptr(wq), ptr(s), ptr(b))
    return wq, s, b


def window_mask(q_len, kv_len, window):
    out = np.zeros((max(q_len, 1), max(kv_len, 1)), dtype=np.uint8)
    if lib().orc_window_mask(q_len, kv_len, window, ptr(out)):
        raise ValueError("invalid mask sizes")
    return out.astype(bool)


def llama3_freqs(theta, factor, lo, hi, orig, head_dim):
    out = np.zeros(head_dim // 2, dtype=np.float32)
    if lib().orc_rope_llama3_freqs(theta, factor, lo, hi, orig, head_dim, ptr(out)):
        raise ValueError("invalid llama3 rope parameters")
    return out


def sample(logits_f32, sp, ctx=None, step=0):
    x = np.ascontiguousarray(logits_f32, dtype=np.float32)
    V = x.shape[-1]
    ctx = np.zeros(0, dtype=np.int32) if ctx is None else np.ascontiguousarray(ctx, dtype=np.int32)
    tok = np.zeros(1, dtype=np.int32)
    lp = np.zeros(1, dtype=np.float32)
    keep = np.zeros(V, dtype=np.uint8)
    lib().orc_sample(ptr(x), V, C.byref(sp), ptr(ctx), len(ctx), step, ptr(tok), ptr(lp), ptr(keep))
    return int(tok[0]), float(lp[0]), keep.astype(bool)


def _filter(fn, x, arg):
    y = np.array(x, dtype=np.float32, copy=True)
    fn(ptr(y), y.shape[-1], arg)
    return y


def top_k(x, k):
    return _filter(lib().orc_top_k, x, k)


def top_p(x, p):
    return _filter(lib().orc_top_p, x, p)


def min_p(x, mp):
    return _filter(lib().orc_min_p, x, mp)


def synth_host_tensors(specs, group, seed=0, std=0.02):
    """The benchmark's seeded weights built on the host by the oracle's copy of
    the generator. specs: (name, kind, rows, cols) as the library's
    synth_tensor_specs gives them; kind "n" is a norm weight of ones."""
    L = lib()
    out = {}
    for i, (name, kind, rows, cols) in enumerate(specs):
        if kind == "n":
            a = np.zeros(rows, np.uint16)
            L.orc_synth_bf16(ptr(a), rows, 0, 0.0, 1.0)
            out[name] = a
            continue
        w = np.zeros((rows, cols // 8), np.uint32)
        s = np.zeros((rows, cols // group), np.uint16)
        b = np.zeros((rows, cols // group), np.uint16)
        if L.orc_synth_quantized(ptr(w), ptr(s), ptr(b), rows, cols, group, seed * 1000003 + i, std):
            raise RuntimeError("orc_synth_quantized: bad shape %s" % name)
        out[name + ".weight"], out[name + ".scales"], out[name + ".biases"] = w, s, b
    return out
