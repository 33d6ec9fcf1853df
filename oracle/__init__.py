"""ctypes bindings for the test oracle.

TEST INFRASTRUCTURE ONLY.  `Oracle` wraps our C restatement of LMc's hot
path (oracle/lmc_oracle.c); `Ref` wraps LMc's own C sources compiled from
source into oracle/_ref/ (oracle/Makefile).  Only tests/, the smoke check in
__graft_entry__ and bench.py's CPU-baseline leg import this package; the
product library never does.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int)


def _ptr(a, t):
    return a.ctypes.data_as(t)


class Oracle:
    """The C restatement (lmc_oracle.c)."""

    def __init__(self, path=None):
        path = path or os.path.join(HERE, "liblmc_oracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        L = self.lib = ctypes.CDLL(path)
        L.orc_block_geometry.argtypes = [ctypes.c_uint32, _i32p, _i32p]
        L.orc_dequant.argtypes = [ctypes.c_uint32, _u8p, _f32p, ctypes.c_size_t]
        L.orc_matmul_vec.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_gelu.argtypes = [ctypes.c_float]
        L.orc_gelu.restype = ctypes.c_float
        L.orc_silu.argtypes = [ctypes.c_float]
        L.orc_silu.restype = ctypes.c_float
        L.orc_softmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int]
        L.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.orc_rope_apply.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int]
        L.orc_rope_cache.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_attention.argtypes = [_f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_sample_top_p.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                       ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_double)]
        L.orc_model_load.argtypes = [ctypes.c_char_p]
        L.orc_model_load.restype = ctypes.c_void_p
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_model_config.argtypes = [ctypes.c_void_p, _i32p]
        L.orc_model_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_model_set_kv.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_kv_q8_row.argtypes = [_f32p, ctypes.c_int, ctypes.POINTER(ctypes.c_int8), ctypes.POINTER(ctypes.c_float)]
        L.orc_kv_round_row.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.orc_f32_to_f16_to_f32.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16_to_f32.restype = ctypes.c_float

    def geometry(self, t):
        be, bb = ctypes.c_int(), ctypes.c_int()
        if self.lib.orc_block_geometry(t, ctypes.byref(be), ctypes.byref(bb)):
            raise ValueError(f"unsupported type {t}")
        return be.value, bb.value

    def dequant(self, t, blocks, n):
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty(n, np.float32)
        if self.lib.orc_dequant(t, _ptr(blocks, _u8p), _ptr(out, _f32p), n):
            raise ValueError("orc_dequant failed")
        return out

    def matmul_vec(self, w, x, bias=None):
        M, K = w.shape
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(M, np.float32)
        b = None if bias is None else _ptr(np.ascontiguousarray(bias, np.float32), _f32p)
        self.lib.orc_matmul_vec(_ptr(out, _f32p), _ptr(w, _f32p), b, _ptr(x, _f32p), M, K)
        return out

    def layer_norm(self, x, w, b):
        x, w, b = (np.ascontiguousarray(a, np.float32) for a in (x, w, b))
        out = np.empty_like(x)
        self.lib.orc_layer_norm(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), _ptr(b, _f32p), x.size)
        return out

    def rms_norm(self, x, w, eps):
        x, w = (np.ascontiguousarray(a, np.float32) for a in (x, w))
        out = np.empty_like(x)
        self.lib.orc_rms_norm(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), x.size, eps)
        return out

    def softmax(self, x):
        x = np.array(x, np.float32)
        self.lib.orc_softmax(_ptr(x, _f32p), x.size)
        return x

    def gelu(self, x):
        return np.array([self.lib.orc_gelu(float(v)) for v in np.ravel(x)], np.float32).reshape(np.shape(x))

    def silu(self, x):
        return np.array([self.lib.orc_silu(float(v)) for v in np.ravel(x)], np.float32).reshape(np.shape(x))

    def rope_cache(self, S, Dh, theta):
        c = np.empty((S, Dh // 2), np.float32)
        s = np.empty((S, Dh // 2), np.float32)
        self.lib.orc_rope_cache(_ptr(c, _f32p), _ptr(s, _f32p), S, Dh, theta)
        return c, s

    def rope_apply(self, vec, cos_row, sin_row):
        v = np.array(vec, np.float32)
        c, s = (np.ascontiguousarray(a, np.float32) for a in (cos_row, sin_row))
        self.lib.orc_rope_apply(_ptr(v, _f32p), _ptr(c, _f32p), _ptr(s, _f32p), v.size)
        return v

    def attention(self, q, kc, vc, H, Hkv, Dh, S, pos):
        q, kc, vc = (np.ascontiguousarray(a, np.float32) for a in (q, kc, vc))
        out = np.empty(H * Dh, np.float32)
        self.lib.orc_attention(_ptr(out, _f32p), _ptr(q, _f32p), _ptr(kc, _f32p), _ptr(vc, _f32p),
                               H, Hkv, Dh, S, pos)
        return out

    def kv_q8_row(self, x):
        """(int8 codes, scale) of one KV row as the int8 cache stores it."""
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.size, np.int8)
        sc = ctypes.c_float()
        self.lib.orc_kv_q8_row(_ptr(x, _f32p), x.size, q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), ctypes.byref(sc))
        return q, sc.value

    def kv_round_rows(self, rows, mode):
        """rows [n][Dh] replaced by what a cache of the given mode returns."""
        r = np.array(rows, np.float32, copy=True).reshape(-1, np.shape(rows)[-1])
        for i in range(r.shape[0]):
            row = np.ascontiguousarray(r[i])
            self.lib.orc_kv_round_row(_ptr(row, _f32p), row.size, mode)
            r[i] = row
        return r.reshape(np.shape(rows))

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return self.lib.orc_argmax(_ptr(x, _f32p), x.size)

    def sample_top_p(self, logits, temperature, top_p, state):
        """(token, next xorshift64 state, margin of the draw to a cdf boundary)."""
        x = np.array(logits, np.float32)
        st, m = ctypes.c_uint64(state), ctypes.c_double()
        tok = self.lib.orc_sample_top_p(_ptr(x, _f32p), x.size, temperature, top_p, ctypes.byref(st), ctypes.byref(m))
        return tok, st.value, m.value

    def model(self, path):
        return OracleModel(self, path)


class OracleModel:
    """orc_model_* : a whole GGUF model dequantized to fp32 on the host."""

    def __init__(self, orc, path):
        self.lib = orc.lib
        self.h = self.lib.orc_model_load(path.encode())
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        c = np.zeros(11, np.int32)
        self.lib.orc_model_config(self.h, _ptr(c, _i32p))
        self.arch, self.V, self.S, self.L, self.H, self.Hkv, self.D, self.F, self.Dh = (int(v) for v in c[:9])

    def set_kv(self, mode):
        """Store K/V rows as a cache of mode 0 (fp32), 1 (fp16) or 2 (int8 rows)."""
        self.lib.orc_model_set_kv(self.h, mode)
        return self

    def forward(self, tok, pos):
        out = np.empty(self.V, np.float32)
        if self.lib.orc_model_forward(self.h, tok, pos, _ptr(out, _f32p)):
            raise ValueError("orc_model_forward failed")
        return out

    def close(self):
        if self.h:
            self.lib.orc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def _has_avx512():
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512bw", "avx512dq", "avx512vl"))


def ref_library_path():
    d = os.path.join(HERE, "_ref")
    if _has_avx512() and os.path.exists(os.path.join(d, "liblmcref_avx512.so")):
        return os.path.join(d, "liblmcref_avx512.so")
    return os.path.join(d, "liblmcref.so")


class Ref:
    """LMc's own compiled sources (oracle/_ref), via ref_shim.c.

    LMc keeps its model in process globals, so one process holds one model.
    """

    def __init__(self, path=None):
        path = path or ref_library_path()
        if not os.path.exists(path):
            raise RuntimeError(f"LMc reference build missing: {path} (run make -C oracle ref)")
        self.path = path
        L = self.lib = ctypes.CDLL(path)
        L.refshim_dequant.argtypes = [ctypes.c_uint32, _u8p, _f32p, ctypes.c_size_t]
        L.refshim_load.argtypes = [ctypes.c_char_p]
        L.refshim_config.argtypes = [_i32p]
        L.refshim_forward.argtypes = [ctypes.c_int, ctypes.c_int, _f32p]
        L.refshim_generate.argtypes = [_i32p, ctypes.c_int, ctypes.c_int, _i32p,
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.refshim_set_threads.argtypes = [ctypes.c_int]
        L.refshim_now.restype = ctypes.c_double
        L.refshim_time_matmul.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.refshim_time_matmul.restype = ctypes.c_double
        L.matmul_vec.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int]
        L.rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.softmax.argtypes = [_f32p, ctypes.c_int]
        L.gelu.argtypes = [ctypes.c_float]
        L.gelu.restype = ctypes.c_float
        L.silu.argtypes = [ctypes.c_float]
        L.silu.restype = ctypes.c_float
        L.rope_apply.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int]
        L.refshim_sample_top_p.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                           ctypes.POINTER(ctypes.c_uint64)]
        self.cfg = None

    def set_threads(self, n):
        self.lib.refshim_set_threads(n)

    def max_threads(self):
        return self.lib.refshim_max_threads()

    def dequant(self, t, blocks, n):
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty(n, np.float32)
        if self.lib.refshim_dequant(t, _ptr(blocks, _u8p), _ptr(out, _f32p), n):
            raise ValueError("unsupported type")
        return out

    def matmul_vec(self, w, x, bias=None):
        M, K = w.shape
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(M, np.float32)
        b = None if bias is None else _ptr(np.ascontiguousarray(bias, np.float32), _f32p)
        self.lib.matmul_vec(_ptr(out, _f32p), _ptr(w, _f32p), b, _ptr(x, _f32p), M, K)
        return out

    def time_matmul(self, w, x, reps, bias=None):
        M, K = w.shape
        out = np.empty(M, np.float32)
        b = None if bias is None else _ptr(bias, _f32p)
        return self.lib.refshim_time_matmul(_ptr(out, _f32p), _ptr(w, _f32p), b, _ptr(x, _f32p), M, K, reps)

    def layer_norm(self, x, w, b):
        x, w, b = (np.ascontiguousarray(a, np.float32) for a in (x, w, b))
        out = np.empty_like(x)
        self.lib.layer_norm(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), _ptr(b, _f32p), x.size)
        return out

    def rms_norm(self, x, w, eps):
        x, w = (np.ascontiguousarray(a, np.float32) for a in (x, w))
        out = np.empty_like(x)
        self.lib.rms_norm(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), x.size, eps)
        return out

    def softmax(self, x):
        x = np.array(x, np.float32)
        self.lib.softmax(_ptr(x, _f32p), x.size)
        return x

    def load(self, path):
        self.lib.refshim_load(path.encode())
        c = np.zeros(9, np.int32)
        self.lib.refshim_config(_ptr(c, _i32p))
        self.cfg = dict(zip(("arch", "V", "S", "L", "H", "Hkv", "D", "F", "Dh"), (int(v) for v in c)))
        return self.cfg

    def forward(self, tok, pos):
        out = np.empty(self.cfg["V"], np.float32)
        self.lib.refshim_forward(tok, pos, _ptr(out, _f32p))
        return out

    def sample_top_p(self, logits, temperature, top_p, state):
        """LMc's own sample_top_p (lmc.c:42-59) from xorshift64 state `state`:
        (token, next state)."""
        x = np.array(logits, np.float32)
        st = ctypes.c_uint64(state)
        tok = self.lib.refshim_sample_top_p(_ptr(x, _f32p), x.size, temperature, top_p, ctypes.byref(st))
        return tok, st.value

    def generate(self, prompt, n_new):
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_new, np.int32)
        tp, td = ctypes.c_double(), ctypes.c_double()
        rc = self.lib.refshim_generate(_ptr(prompt, _i32p), prompt.size, n_new, _ptr(ids, _i32p),
                                       ctypes.byref(tp), ctypes.byref(td))
        if rc:
            raise ValueError("context overflow")
        return ids, tp.value, td.value
