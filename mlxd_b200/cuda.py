"""ctypes binding of libmlxd_cuda (include/mlxd_cuda.h).

This is the Python mirror of the reference's engine-side calls for the decoder
step: model load (src/engine/emodel.c:176-211), model_forward
(emodel.c:221-337), the KV cache (src/engine/kvcache.h), the sampler
(src/engine/sampler.h) and the generate loop (src/engine/engine.c:360-602).
Every call goes through the C ABI into the sm_100a kernels; there is no CPU
path, and importing fails loudly when the library has not been built.
"""
import ctypes as C
import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmlxd_cuda.so")

BF16, F32, U32, I32 = 1, 2, 3, 4
QWEN3, LLAMA, MISTRAL, QWEN3_5 = 1, 2, 3, 4


class ModelConfig(C.Structure):
    _fields_ = [("family", C.c_int), ("vocab", C.c_int), ("hidden", C.c_int),
                ("layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("max_pos", C.c_int),
                ("eps", C.c_float), ("rope_theta", C.c_float), ("qk_norm", C.c_int),
                ("tie", C.c_int), ("attn_gate", C.c_int), ("rope_dims", C.c_int),
                ("rope_llama3", C.c_int), ("rope_factor", C.c_float),
                ("rope_lo", C.c_float), ("rope_hi", C.c_float), ("rope_orig_max", C.c_int),
                ("window", C.c_int), ("qbits", C.c_int), ("qgroup", C.c_int),
                ("n_eos", C.c_int), ("eos", C.c_int * 8), ("tp_rank", C.c_int),
                ("tp_size", C.c_int)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p), ("on_device", C.c_int)]


class Sampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("min_p", C.c_float), ("seed", C.c_int),
                ("repetition_penalty", C.c_float), ("repetition_context", C.c_int)]


def sampling(temperature=1.0, top_p=1.0, top_k=-1, min_p=0.0, seed=-1,
             repetition_penalty=1.0, repetition_context=20):
    """SAMPLING_PARAMS_DEFAULT (src/core/types.h:34-35) plus the repetition
    penalty (off at 1.0)."""
    return Sampling(temperature, top_p, top_k, min_p, seed, repetition_penalty,
                    repetition_context)


PREFILL_HOOK = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_int)
STEP_HOOK = C.CFUNCTYPE(None, C.c_void_p, C.c_int)
SEED_HOOK = C.CFUNCTYPE(None, C.c_void_p)


class GenControl(C.Structure):
    """mlxd_gen_control: cancel/shutdown flags and the three generate hooks
    (engine_gen_hooks_t)."""
    _fields_ = [("shutdown", C.POINTER(C.c_int)), ("cancelled", C.POINTER(C.c_int)),
                ("on_prefill_chunk", PREFILL_HOOK), ("on_decode_step", STEP_HOOK),
                ("on_before_seed", SEED_HOOK), ("ud", C.c_void_p), ("stopped", C.c_int)]


def gen_control(on_prefill_chunk=None, on_decode_step=None, on_before_seed=None):
    """A control block with its own flags (ctl.flags = (shutdown, cancelled),
    c_int objects the caller sets) and Python hooks."""
    sd, cn = C.c_int(0), C.c_int(0)
    ctl = GenControl(C.pointer(sd), C.pointer(cn),
                     PREFILL_HOOK(lambda ud, pos, n: on_prefill_chunk(pos, n)) if on_prefill_chunk
                     else PREFILL_HOOK(),
                     STEP_HOOK(lambda ud, step: on_decode_step(step)) if on_decode_step else STEP_HOOK(),
                     SEED_HOOK(lambda ud: on_before_seed()) if on_before_seed else SEED_HOOK(), None, 0)
    ctl.flags = (sd, cn)
    return ctl


# symbol -> (restype, argtypes)
P = C.c_void_p
_SIGS = {
    "mlxd_cuda_last_error": (C.c_char_p, []),
    "mlxd_cuda_init": (C.c_int, [C.c_int]),
    "mlxd_cuda_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "mlxd_cuda_stream_create": (C.c_int, [C.POINTER(P)]),
    "mlxd_cuda_stream_destroy": (C.c_int, [P]),
    "mlxd_cuda_synchronize": (C.c_int, [P]),
    "mlxd_cuda_alloc": (C.c_int, [C.POINTER(P), C.c_size_t]),
    "mlxd_cuda_free": (C.c_int, [P]),
    "mlxd_cuda_upload": (C.c_int, [P, P, C.c_size_t, P]),
    "mlxd_cuda_download": (C.c_int, [P, P, C.c_size_t, P]),
    "mlxd_cuda_memset": (C.c_int, [P, C.c_int, C.c_size_t, P]),
    "mlxd_cuda_active_memory": (C.c_size_t, []),
    "mlxd_cuda_peak_memory": (C.c_size_t, []),
    "mlxd_cuda_model_create": (C.c_int, [C.POINTER(P), C.POINTER(ModelConfig),
                                         C.POINTER(Tensor), C.c_int]),
    "mlxd_cuda_model_destroy": (None, [P]),
    "mlxd_cuda_model_weight_bytes": (C.c_size_t, [P]),
    "mlxd_cuda_model_tp_init": (C.c_int, [P, P]),
    "mlxd_cuda_nccl_unique_id": (C.c_int, [P]),
    "mlxd_cuda_tp_plan": (C.c_int, [C.POINTER(ModelConfig), C.c_int, C.c_int, P]),
    "mlxd_cuda_kv_create": (C.c_int, [C.POINTER(P), P, C.c_int]),
    "mlxd_cuda_kv_destroy": (None, [P]),
    "mlxd_cuda_kv_offset": (C.c_int, [P, C.c_int]),
    "mlxd_cuda_kv_capacity": (C.c_int, [P, C.c_int]),
    "mlxd_cuda_kv_reset": (C.c_int, [P]),
    "mlxd_cuda_kv_read": (C.c_int, [P, C.c_int, C.c_int, P, C.POINTER(C.c_int)]),
    "mlxd_cuda_forward": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, P, P]),
    "mlxd_cuda_linear_create": (C.c_int, [C.POINTER(P), P, P, P, C.c_int, C.c_int, C.c_int,
                                          C.c_int, C.c_int]),
    "mlxd_cuda_linear_destroy": (None, [P]),
    "mlxd_cuda_linear": (C.c_int, [P, P, C.c_int, P, P]),
    "mlxd_cuda_linear_noalloc": (C.c_int, [P, P, P, P]),
    "mlxd_cuda_linear_timed": (C.c_int, [C.POINTER(P), C.c_int, C.c_int, P, P,
                                         C.POINTER(C.c_float)]),
    "mlxd_cuda_linear_timed_chained": (C.c_int, [C.POINTER(P), C.c_int, C.c_int, P, P,
                                                 C.POINTER(C.c_float)]),
    "mlxd_cuda_rmsnorm": (C.c_int, [P, C.c_int, C.c_int, P, C.c_float, P, P]),
    "mlxd_cuda_sample": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(Sampling), P, C.c_int,
                                   C.c_uint64, P, P, P, P]),
    "mlxd_cuda_generate": (C.c_int, [P, P, P, C.c_int, C.c_int, C.POINTER(Sampling), C.c_int,
                                     P, P, P]),
    "mlxd_cuda_generate_ctl": (C.c_int, [P, P, P, C.c_int, C.c_int, C.POINTER(Sampling), C.c_int,
                                         P, P, P, C.POINTER(GenControl)]),
    "mlxd_cuda_step_async": (C.c_int, [P, P, P, C.POINTER(Sampling), P, C.c_int, C.c_uint64, P, P, P]),
    "mlxd_cuda_read_token": (C.c_int, [P, P, P]),
    "mlxd_cuda_kv_write": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, P]),
    "mlxd_cuda_kv_gather": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P]),
    "mlxd_cuda_kv_set_offset": (C.c_int, [P, C.c_int, P]),
    "mlxd_cuda_synth_quantized": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                            C.c_float, P]),
    "mlxd_cuda_synth_bf16": (C.c_int, [P, C.c_size_t, C.c_uint64, C.c_float, C.c_float, P]),
    "mlxd_host_synth_quantized": (None, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                         C.c_float]),
    "mlxd_host_synth_bf16": (None, [P, C.c_size_t, C.c_uint64, C.c_float, C.c_float]),
}

_lib = None


def lib():
    """Load libmlxd_cuda; raises if it is missing (no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libmlxd_cuda.so not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class CudaError(RuntimeError):
    pass


def check(rc, what=""):
    if rc != 0:
        msg = lib().mlxd_cuda_last_error().decode(errors="replace")
        raise CudaError(f"{what}: {msg}")


def ptr(a):
    return C.c_void_p(a.ctypes.data)


# ------------------------------------------------------------ device memory

class DeviceBuffer:
    """A device allocation owned by Python (mlxd_cuda_alloc / _free)."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        check(lib().mlxd_cuda_alloc(C.byref(p), max(self.nbytes, 16)), "alloc")
        self.ptr = p

    @classmethod
    def from_array(cls, a):
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        if a.nbytes:
            check(lib().mlxd_cuda_upload(b.ptr, ptr(a), a.nbytes, None), "upload")
        return b

    def to_array(self, dtype, shape):
        out = np.empty(shape, dtype=dtype)
        if out.nbytes:
            check(lib().mlxd_cuda_download(ptr(out), self.ptr, out.nbytes, None), "download")
        return out

    def zero(self):
        check(lib().mlxd_cuda_memset(self.ptr, 0, self.nbytes, None), "memset")
        check(lib().mlxd_cuda_synchronize(None), "sync")

    def free(self):
        if self.ptr:
            lib().mlxd_cuda_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def init(device=0):
    check(lib().mlxd_cuda_init(device), "init")


def synchronize():
    check(lib().mlxd_cuda_synchronize(None), "synchronize")


# --------------------------------------------------------------- checkpoints

_ST_DT = {"BF16": (BF16, np.uint16), "F32": (F32, np.float32), "U32": (U32, np.uint32)}


def read_safetensors(path):
    """8-byte little-endian header length, JSON header, raw tensors."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, meta in hdr.items():
            if name == "__metadata__":
                continue
            _, npdt = _ST_DT[meta["dtype"]]
            a, b = meta["data_offsets"]
            f.seek(base + a)
            out[name] = np.frombuffer(f.read(b - a), dtype=npdt).reshape(meta["shape"]).copy()
        return out


def read_checkpoint(model_dir):
    """Single file or index-guided shard set (weights.c:32-192)."""
    idx = os.path.join(model_dir, "model.safetensors.index.json")
    files = (sorted(set(json.load(open(idx))["weight_map"].values())) if os.path.exists(idx)
             else ["model.safetensors"])
    t = {}
    for fn in files:
        t.update(read_safetensors(os.path.join(model_dir, fn)))
    return t


def tp_plan(cfg, rank, size):
    """The library's tensor-parallel shard plan (host only): {name: (row0,
    rows, col0, cols)} of this rank's part of each full projection."""
    r = np.zeros(32, np.int32)
    check(lib().mlxd_cuda_tp_plan(C.byref(cfg), rank, size, ptr(r)), "tp_plan")
    names = ["q", "k", "v", "o", "gate", "up", "down", "lm_head"]
    return {n: tuple(int(v) for v in r[4 * i:4 * i + 4]) for i, n in enumerate(names)}


def config_from_json(cj, tp_rank=0, tp_size=1):
    """model_config_load (src/model/model.c:667-1031) for the dense families on
    the path: qwen3 / llama / mistral / qwen3_5 defaults."""
    fam = {"qwen3": QWEN3, "llama": LLAMA, "mistral": MISTRAL, "qwen3_5": QWEN3_5,
           "qwen3_5_text": QWEN3_5}.get(cj.get("model_type"))
    if fam is None:
        raise ValueError("unsupported model family %r" % cj.get("model_type"))
    c = ModelConfig()
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
    theta, prf = cj.get("rope_theta", 1e6), 1.0
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
    if isinstance(rs, dict):
        rt = rs.get("rope_type") or rs.get("type")
        if fam == QWEN3 and rt is not None:
            raise ValueError("RoPE scaling not supported for qwen3")
        if rt == "llama3":
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
    c.n_eos = min(len(eos), 8)
    for i, e in enumerate(eos[:8]):
        c.eos[i] = e
    c.tp_rank, c.tp_size = tp_rank, tp_size
    return c


# ------------------------------------------------------------------- model

class Model:
    """engine_model_t over libmlxd_cuda (src/engine/emodel.h:11-28)."""

    def __init__(self, cfg, tensors, on_device=False):
        self.cfg = cfg
        names = list(tensors.keys())
        arr = (Tensor * len(names))()
        self._keep = []
        for i, n in enumerate(names):
            t = tensors[n]
            nb = n.encode()
            self._keep.append(nb)
            if on_device:
                dbuf, dt, shape = t
                arr[i].data = dbuf.ptr
                arr[i].on_device = 1
            else:
                t = np.ascontiguousarray(t)
                self._keep.append(t)
                dt = {np.uint16: BF16, np.float32: F32, np.uint32: U32}[t.dtype.type]
                shape = t.shape
                arr[i].data = t.ctypes.data
                arr[i].on_device = 0
            arr[i].name = nb
            arr[i].dtype = dt
            arr[i].ndim = len(shape)
            for j, s in enumerate(shape):
                arr[i].shape[j] = s
        m = C.c_void_p()
        check(lib().mlxd_cuda_model_create(C.byref(m), C.byref(cfg), arr, len(names)),
              "model_create")
        self._keep = None
        self.m = m
        self.vocab_local = cfg.vocab // max(cfg.tp_size, 1)

    @classmethod
    def from_dir(cls, model_dir, tp_rank=0, tp_size=1):
        cj = json.load(open(os.path.join(model_dir, "config.json")))
        return cls(config_from_json(cj, tp_rank, tp_size), read_checkpoint(model_dir))

    def weight_bytes(self):
        return lib().mlxd_cuda_model_weight_bytes(self.m)

    def tp_init(self, uid_bytes):
        buf = C.create_string_buffer(bytes(uid_bytes), 128)
        check(lib().mlxd_cuda_model_tp_init(self.m, buf), "tp_init")

    def new_kv(self, capacity):
        return KVCache(self, capacity)

    def forward(self, kv, ids, want_logits=True, logits=None):
        """model_forward: returns the last position's bf16 logits (uint16 bits)
        as a numpy array, or writes them to the given DeviceBuffer."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        own = logits is None and want_logits
        if own:
            logits = DeviceBuffer(self.vocab_local * 2)
        check(lib().mlxd_cuda_forward(self.m, kv.kv, ptr(ids), len(ids), 0, int(want_logits),
                                      logits.ptr if want_logits else None, None), "forward")
        if own:
            return logits.to_array(np.uint16, (self.vocab_local,))
        return None

    def generate(self, prompt, max_new, sp=None, chunk=512, kv=None, logprobs=False, control=None):
        """handle_generate_real: returns (tokens, logprobs or None, timing dict).
        control: a gen_control() block (cancel/shutdown flags and hooks)."""
        sp = sp or sampling(temperature=0.0)
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        own_kv = kv is None
        if own_kv:
            kv = self.new_kv(len(prompt) + max_new + 1)
        out = np.zeros(max_new, dtype=np.int32)
        lps = np.zeros(max_new, dtype=np.float32) if logprobs else None
        timing = np.zeros(4 + max_new, dtype=np.float64)
        n = lib().mlxd_cuda_generate_ctl(self.m, kv.kv, ptr(prompt), len(prompt), max_new,
                                         C.byref(sp), chunk, ptr(out),
                                         ptr(lps) if logprobs else None, ptr(timing),
                                         C.byref(control) if control is not None else None)
        if n < 0:
            check(-1, "generate")
        t = {"prefill_ms": timing[0], "decode_ms": timing[1], "decode_steps": timing[2],
             "decode_wall_ms": timing[3], "step_end_ms": timing[4:4 + n].copy()}
        return out[:n], (lps[:n] if logprobs else None), t

    def close(self):
        if getattr(self, "m", None):
            lib().mlxd_cuda_model_destroy(self.m)
            self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """kvcache_t over libmlxd_cuda (src/engine/kvcache.h:11-51)."""

    def __init__(self, model, capacity):
        self.model = model
        kv = C.c_void_p()
        check(lib().mlxd_cuda_kv_create(C.byref(kv), model.m, capacity), "kv_create")
        self.kv = kv

    def offset(self, layer=0):
        return lib().mlxd_cuda_kv_offset(self.kv, layer)

    def capacity(self, layer=0):
        return lib().mlxd_cuda_kv_capacity(self.kv, layer)

    def reset(self):
        check(lib().mlxd_cuda_kv_reset(self.kv), "kv_reset")

    def read(self, layer, value=False):
        c = self.model.cfg
        hkv = c.n_kv_heads // max(c.tp_size, 1)
        cap = self.capacity(layer)
        buf = np.zeros((hkv, cap, c.head_dim), dtype=np.uint16)
        n = C.c_int()
        check(lib().mlxd_cuda_kv_read(self.kv, layer, int(value), ptr(buf), C.byref(n)), "kv_read")
        return np.ascontiguousarray(buf.reshape(-1)[: hkv * n.value * c.head_dim]).reshape(
            hkv, n.value, c.head_dim)

    def close(self):
        if getattr(self, "kv", None):
            lib().mlxd_cuda_kv_destroy(self.kv)
            self.kv = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Linear:
    """One quantized projection in the tile layout (fwd_linear's triplet)."""

    def __init__(self, w, scales, biases, group, rows=None, cols=None, sdtype=BF16):
        if isinstance(w, DeviceBuffer):
            h = C.c_void_p()
            check(lib().mlxd_cuda_linear_create(C.byref(h), w.ptr, scales.ptr, biases.ptr,
                                                sdtype, rows, cols, group, 1), "linear_create")
            self.h, self.rows, self.cols = h, rows, cols
            return
        sdt = F32 if scales.dtype == np.float32 else BF16
        rows, cols = w.shape[0], w.shape[1] * 8
        h = C.c_void_p()
        w, scales, biases = (np.ascontiguousarray(a) for a in (w, scales, biases))
        check(lib().mlxd_cuda_linear_create(C.byref(h), ptr(w), ptr(scales), ptr(biases), sdt,
                                            rows, cols, group, 0), "linear_create")
        self.h, self.rows, self.cols = h, rows, cols

    def __call__(self, x_bf16):
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        S = 1 if x.ndim == 1 else x.shape[0]
        dx = DeviceBuffer.from_array(x)
        dy = DeviceBuffer(S * self.rows * 2)
        check(lib().mlxd_cuda_linear(self.h, dx.ptr, S, dy.ptr, None), "linear")
        return dy.to_array(np.uint16, (S, self.rows))

    def close(self):
        if getattr(self, "h", None):
            lib().mlxd_cuda_linear_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def linear_timed(linears, iters, x_dev, y_dev, chained=False):
    """Mean ms per decode-GEMV launch over round-robin launches; chained:
    each launch chained to the previous one by programmatic dependent launch
    (the decode graph's launch mode)."""
    arr = (C.c_void_p * len(linears))(*[l.h.value for l in linears])
    ms = C.c_float()
    fn = lib().mlxd_cuda_linear_timed_chained if chained else lib().mlxd_cuda_linear_timed
    check(fn(arr, len(linears), iters, x_dev.ptr, y_dev.ptr, C.byref(ms)), "linear_timed")
    return ms.value


def rmsnorm(x_bf16, w_bf16, eps):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    n = x.shape[-1]
    rows = x.size // n
    dx, dw = DeviceBuffer.from_array(x), DeviceBuffer.from_array(np.ascontiguousarray(w_bf16))
    dy = DeviceBuffer(x.nbytes)
    check(lib().mlxd_cuda_rmsnorm(dx.ptr, rows, n, dw.ptr, eps, dy.ptr, None), "rmsnorm")
    return dy.to_array(np.uint16, x.shape)


def sample(logits, sp, ctx=None, step=0):
    """sampler_sample_lazy on one row: returns (token, logprob, keep mask)."""
    x = np.ascontiguousarray(logits)
    dt = BF16 if x.dtype == np.uint16 else F32
    if dt == F32:
        x = x.astype(np.float32)
    V = x.shape[-1]
    dl = DeviceBuffer.from_array(x)
    ctx = np.zeros(1, np.int32) if ctx is None or len(ctx) == 0 else np.asarray(ctx, np.int32)
    n_ctx = 0 if ctx is None else len(ctx)
    dc = DeviceBuffer.from_array(ctx)
    dt_tok, dlp, dkeep = DeviceBuffer(4), DeviceBuffer(4), DeviceBuffer(V)
    check(lib().mlxd_cuda_sample(dl.ptr, dt, V, C.byref(sp), dc.ptr, n_ctx, step, dt_tok.ptr,
                                 dlp.ptr, dkeep.ptr, None), "sample")
    synchronize()
    tok = int(dt_tok.to_array(np.int32, (1,))[0])
    lp = float(dlp.to_array(np.float32, (1,))[0])
    keep = dkeep.to_array(np.uint8, (V,)).astype(bool)
    return tok, lp, keep


# ----------------------------------------------------------- synthetic models

def synth_config(hidden, layers, n_heads, n_kv_heads, head_dim, inter, vocab, family=QWEN3,
                 tie=False, window=0, max_pos=4096, group=64, theta=1e6, llama3=None,
                 eps=1e-6, tp_rank=0, tp_size=1):
    c = ModelConfig()
    c.family = family
    c.vocab, c.hidden, c.layers = vocab, hidden, layers
    c.n_heads, c.n_kv_heads, c.head_dim, c.inter = n_heads, n_kv_heads, head_dim, inter
    c.max_pos = max_pos
    c.eps, c.rope_theta = eps, theta
    c.qk_norm = 1 if family in (QWEN3, QWEN3_5) else 0
    c.tie = int(tie)
    c.rope_dims = head_dim
    if llama3:
        c.rope_llama3 = 1
        c.rope_factor, c.rope_lo, c.rope_hi, c.rope_orig_max = llama3
    c.window = window
    c.qbits, c.qgroup = 4, group
    c.tp_rank, c.tp_size = tp_rank, tp_size
    return c


def synth_tensor_specs(cfg):
    """(name, kind, rows, cols) of every tensor of a dense decoder checkpoint."""
    H, D = cfg.hidden, cfg.head_dim
    q = cfg.n_heads * D * (2 if cfg.attn_gate else 1)
    kvd = cfg.n_kv_heads * D
    specs = [("model.embed_tokens", "q", cfg.vocab, H), ("model.norm.weight", "n", H, 0)]
    if not cfg.tie:
        specs.append(("lm_head", "q", cfg.vocab, H))
    for l in range(cfg.layers):
        p = "model.layers.%d." % l
        specs += [(p + "self_attn.q_proj", "q", q, H), (p + "self_attn.k_proj", "q", kvd, H),
                  (p + "self_attn.v_proj", "q", kvd, H),
                  (p + "self_attn.o_proj", "q", H, cfg.n_heads * D),
                  (p + "mlp.gate_proj", "q", cfg.inter, H), (p + "mlp.up_proj", "q", cfg.inter, H),
                  (p + "mlp.down_proj", "q", H, cfg.inter),
                  (p + "input_layernorm.weight", "n", H, 0),
                  (p + "post_attention_layernorm.weight", "n", H, 0)]
        if cfg.qk_norm:
            specs += [(p + "self_attn.q_norm.weight", "n", D, 0),
                      (p + "self_attn.k_norm.weight", "n", D, 0)]
    return specs


def synth_host_tensors(cfg, seed=0, std=0.02):
    """Seeded MLX-format tensors in host memory (small configs)."""
    L = lib()
    out = {}
    for i, (name, kind, rows, cols) in enumerate(synth_tensor_specs(cfg)):
        if kind == "n":
            a = np.zeros(rows, np.uint16)
            L.mlxd_host_synth_bf16(ptr(a), rows, 0, 0.0, 1.0)
            out[name] = a
            continue
        G = cfg.qgroup
        w = np.zeros((rows, cols // 8), np.uint32)
        s = np.zeros((rows, cols // G), np.uint16)
        b = np.zeros((rows, cols // G), np.uint16)
        L.mlxd_host_synth_quantized(ptr(w), ptr(s), ptr(b), rows, cols, G, seed * 1000003 + i, std)
        out[name + ".weight"], out[name + ".scales"], out[name + ".biases"] = w, s, b
    return out


def synth_device_tensors(cfg, seed=0, std=0.02):
    """Seeded MLX-format tensors generated on the GPU (full-size configs);
    identical bits to synth_host_tensors. Returns name -> (DeviceBuffer, dtype, shape)."""
    L = lib()
    out = {}
    for i, (name, kind, rows, cols) in enumerate(synth_tensor_specs(cfg)):
        if kind == "n":
            d = DeviceBuffer(rows * 2)
            check(L.mlxd_cuda_synth_bf16(d.ptr, rows, 0, 0.0, 1.0, None), "synth")
            out[name] = (d, BF16, (rows,))
            continue
        G = cfg.qgroup
        w = DeviceBuffer(rows * cols // 2)
        s = DeviceBuffer(rows * (cols // G) * 2)
        b = DeviceBuffer(rows * (cols // G) * 2)
        check(L.mlxd_cuda_synth_quantized(w.ptr, s.ptr, b.ptr, rows, cols, G, seed * 1000003 + i,
                                          std, None), "synth")
        out[name + ".weight"] = (w, U32, (rows, cols // 8))
        out[name + ".scales"] = (s, BF16, (rows, cols // G))
        out[name + ".biases"] = (b, BF16, (rows, cols // G))
    synchronize()
    return out


def device_tensors_to_host(dev):
    np_dt = {BF16: np.uint16, F32: np.float32, U32: np.uint32}
    return {n: buf.to_array(np_dt[dt], shape) for n, (buf, dt, shape) in dev.items()}


def synth_prompt(n, vocab, seed=0):
    """Uniform prompt ids from SplitMix64 on a separate stream."""
    out = np.zeros(n, np.int64)
    z = (seed * 0x9E3779B97F4A7C15 + 0x70726F6D) & 0xFFFFFFFFFFFFFFFF
    for i in range(n):
        z = (z + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        x = z
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 31
        out[i] = x % vocab
    return out.astype(np.int32)
