"""ctypes bindings for liblmc_b200.so (the C ABI in include/lmc_cuda.h).

The library is the product; these bindings only marshal pointers.  Device
buffers may be any object with a device address (torch CUDA tensors are used
by the tests and the bench for convenience).  Loading fails loudly when the
shared object is missing: there is no CPU path behind any of these calls.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblmc_b200.so")

LMC_OK = 0
EPI_NONE, EPI_GELU, EPI_ACCUM = 0, 1, 2
KV_F32, KV_F16, KV_Q8 = 0, 1, 2

_c = ctypes
_vp, _i, _u32, _sz, _f = _c.c_void_p, _c.c_int, _c.c_uint32, _c.c_size_t, _c.c_float
_ip = _c.POINTER(_c.c_int)

SIGNATURES = {
    "lmc_last_error": ([], _c.c_char_p),
    "lmc_init": ([_i], _i),
    "lmc_device_status": ([], _i),
    "lmc_block_geometry": ([_u32, _ip, _ip], _i),
    "lmc_dequant": ([_u32, _vp, _sz, _vp, _vp], _i),
    "lmc_qtensor_upload": ([_u32, _i, _i, _vp, _sz, _c.POINTER(_vp)], _i),
    "lmc_qtensor_free": ([_vp], _i),
    "lmc_qtensor_blocks": ([_vp], _vp),
    "lmc_qtensor_has_tiled": ([_vp], _i),
    "lmc_matmul": ([_vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp], _i),
    "lmc_matmul_kernel": ([_vp, _i, _i], ctypes.c_char_p),
    "lmc_matmul_blocks": ([_u32, _vp, _i, _i, _vp, _i, _vp, _vp, _i, _i, _i, _vp], _i),
    "lmc_layer_norm": ([_vp, _vp, _vp, _vp, _i, _i, _vp], _i),
    "lmc_rms_norm": ([_vp, _vp, _vp, _i, _i, _f, _vp], _i),
    "lmc_softmax": ([_vp, _i, _i, _vp], _i),
    "lmc_gelu": ([_vp, _sz, _vp], _i),
    "lmc_silu": ([_vp, _sz, _vp], _i),
    "lmc_swiglu": ([_vp, _vp, _sz, _vp], _i),
    "lmc_rope_apply": ([_vp, _vp, _vp, _i, _i, _vp], _i),
    "lmc_argmax": ([_vp, _i, _i, _vp, _vp], _i),
    "lmc_attention_workspace_bytes": ([_i, _i, _i, _i], _sz),
    "lmc_attention_decode": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp], _i),
    "lmc_attention_decode_noalloc": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _vp], _i),
    "lmc_attention_decode_paged": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _i, _i, _i, _vp, _sz,
                                    _vp], _i),
    "lmc_model_load": ([_c.c_char_p, _i, _i, _c.POINTER(_vp)], _i),
    "lmc_nccl_unique_id": ([_vp], _i),
    "lmc_model_load_tp": ([_c.c_char_p, _i, _i, _i, _i, _vp, _c.POINTER(_vp)], _i),
    "lmc_model_load_ex": ([_c.c_char_p, _i, _i, _i, _i, _i, _vp, _c.POINTER(_vp)], _i),
    "lmc_model_load_paged": ([_c.c_char_p, _i, _i, _i, _i, _i, _i, _i, _vp, _c.POINTER(_vp)], _i),
    "lmc_model_release_seq": ([_vp, _i], _i),
    "lmc_model_kv_pages": ([_vp, _ip, _ip, _ip], _i),
    "lmc_model_prefill": ([_vp, _i, _ip, _i, _i, _vp, _ip], _i),
    "lmc_model_shard": ([_vp, _ip, _ip, _ip, _ip], _i),
    "lmc_model_get_config": ([_vp, _vp], _i),
    "lmc_model_free": ([_vp], _i),
    "lmc_model_forward": ([_vp, _ip, _ip, _i, _vp, _ip], _i),
    "lmc_model_generate": ([_vp, _ip, _i, _i, _i, _i, _ip], _i),
    "lmc_model_replay": ([_vp, _i, _vp], _i),
    "lmc_model_device_buffer": ([_vp, _i], _vp),
    "lmc_model_graph_kernels": ([_vp], _i),
    "lmc_qtensor_shape": ([_vp, _c.POINTER(_u32), _ip, _ip], _i),
    "lmc_buffer_alloc": ([_sz, _c.POINTER(_vp)], _i),
    "lmc_buffer_free": ([_vp], _i),
    "lmc_copy": ([_vp, _vp, _sz, _i, _vp], _i),
    "lmc_stream_sync": ([_vp], _i),
    "lmc_model_matrix": ([_vp, _i, _i], _vp),
    "lmc_model_vector": ([_vp, _i, _i, _ip], _vp),
    "lmc_sample_top_p": ([_vp, _i, _i, _f, _f, _vp, _vp, _vp], _i),
    "lmc_rng_seed": ([_c.c_uint64], _c.c_uint64),
    "lmc_model_generate_sample": ([_vp, _ip, _i, _i, _i, _f, _f, _c.c_uint64, _i, _ip], _i),
    "lmc_set_wait_limit": ([_c.c_longlong], _i),
    "lmc_wait_selftest": ([_i], _i),
}


class LmcError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"lmc error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Load liblmc_b200.so once (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C lmc_b200` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc):
    if rc != LMC_OK:
        raise LmcError(rc, lib().lmc_last_error().decode(errors="replace"))
    return rc


def call(name, *args):
    return check(getattr(lib(), name)(*args))


def ptr(t):
    """Device (or host) address of a tensor / array, or None."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    return int(t)


class ModelConfig(ctypes.Structure):
    _fields_ = [("arch", _i), ("vocab_size", _i), ("seq_len", _i), ("n_layers", _i), ("n_heads", _i),
                ("n_kv_heads", _i), ("embed_dim", _i), ("ffn_dim", _i), ("head_dim", _i),
                ("rope_theta", _f), ("norm_eps", _f)]


class QTensor:
    """A quantized matrix on the device (lmc_qtensor_upload)."""

    def __init__(self, qtype, rows, cols, blocks):
        import numpy as np
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        h = _vp()
        call("lmc_qtensor_upload", qtype, rows, cols, blocks.ctypes.data, blocks.nbytes, ctypes.byref(h))
        self.h, self.qtype, self.rows, self.cols = h, qtype, rows, cols

    @property
    def tiled(self):
        return bool(lib().lmc_qtensor_has_tiled(self.h))

    def matmul(self, x, y, batch=1, bias=None, epilogue=EPI_NONE, ldx=None, ldy=None, stream=None):
        call("lmc_matmul", self.h, ptr(x), ldx or self.cols, ptr(bias), ptr(y), ldy or self.rows, batch,
             epilogue, stream)

    def close(self):
        if self.h:
            lib().lmc_qtensor_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id():
    """128-byte NCCL group id (lmc_nccl_unique_id), made on one rank and
    handed to every rank of a tensor-parallel group."""
    buf = ctypes.create_string_buffer(128)
    call("lmc_nccl_unique_id", ctypes.cast(buf, _vp))
    return buf.raw


class Model:
    """A GGUF model loaded onto the device (lmc_model_load), or one
    tensor-parallel shard of it when tp = (rank, size, nccl_id) is given
    (lmc_model_load_tp; every rank of the group constructs its shard).
    max_rows > max_batch: rows per step for prefill() chunks (lmc_model_load_ex).
    page_size: a paged KV cache of n_pages pages (lmc_model_load_paged)."""

    def __init__(self, path, max_batch=1, kv_dtype=KV_F32, tp=None, max_rows=None, page_size=0, n_pages=0):
        h = _vp()
        if page_size:
            rank, size, nid = tp if tp is not None else (0, 1, None)
            idbuf = ctypes.create_string_buffer(bytes(nid), 128) if nid is not None else None
            call("lmc_model_load_paged", path.encode(), max_batch, max(max_rows or 0, max_batch), kv_dtype,
                 page_size, n_pages, rank, size, ctypes.cast(idbuf, _vp) if idbuf is not None else None,
                 ctypes.byref(h))
        elif max_rows is not None and max_rows > max_batch:
            rank, size, nid = tp if tp is not None else (0, 1, None)
            idbuf = ctypes.create_string_buffer(bytes(nid), 128) if nid is not None else None
            call("lmc_model_load_ex", path.encode(), max_batch, max_rows, kv_dtype, rank, size,
                 ctypes.cast(idbuf, _vp) if idbuf is not None else None, ctypes.byref(h))
        elif tp is None:
            call("lmc_model_load", path.encode(), max_batch, kv_dtype, ctypes.byref(h))
        else:
            rank, size, nid = tp
            idbuf = ctypes.create_string_buffer(bytes(nid), 128)
            call("lmc_model_load_tp", path.encode(), max_batch, kv_dtype, rank, size, ctypes.cast(idbuf, _vp),
                 ctypes.byref(h))
        self.h = h
        self.cfg = ModelConfig()
        call("lmc_model_get_config", self.h, ctypes.byref(self.cfg))
        self.max_batch = max_batch
        r, n, v0, vl = (ctypes.c_int() for _ in range(4))
        call("lmc_model_shard", self.h, ctypes.byref(r), ctypes.byref(n), ctypes.byref(v0), ctypes.byref(vl))
        self.tp_rank, self.tp_size, self.vocab_begin, self.vocab_rows = r.value, n.value, v0.value, vl.value

    def forward(self, tokens, positions, want_logits=True):
        import numpy as np
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        B = tokens.size
        logits = np.empty((B, self.vocab_rows), np.float32) if want_logits else None
        nxt = np.empty(B, np.int32)
        call("lmc_model_forward", self.h, tokens.ctypes.data_as(_ip), positions.ctypes.data_as(_ip), B,
             None if logits is None else logits.ctypes.data, nxt.ctypes.data_as(_ip))
        return logits, nxt

    def prefill(self, seq, tokens, start_pos=0, want_logits=True):
        """Batched prefill of sequence `seq` (lmc_model_prefill): tokens at
        positions start_pos.. -> (last position's logits or None, next id)."""
        import numpy as np
        tokens = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.vocab_rows, np.float32) if want_logits else None
        nxt = np.empty(1, np.int32)
        call("lmc_model_prefill", self.h, seq, tokens.ctypes.data_as(_ip), tokens.size, start_pos,
             None if logits is None else logits.ctypes.data, nxt.ctypes.data_as(_ip))
        return logits, int(nxt[0])

    def generate(self, prompt, n_new, use_graph=True):
        """prompt: [B][n_prompt] token ids -> [B][n_new] greedy ids."""
        import numpy as np
        prompt = np.ascontiguousarray(np.atleast_2d(prompt), np.int32)
        B, n_prompt = prompt.shape
        out = np.empty((B, n_new), np.int32)
        call("lmc_model_generate", self.h, prompt.ctypes.data_as(_ip), n_prompt, B, n_new, int(use_graph),
             out.ctypes.data_as(_ip))
        return out

    def release_seq(self, seq):
        """Give sequence `seq`'s KV pages back to the pool (lmc_model_release_seq)."""
        call("lmc_model_release_seq", self.h, seq)

    def kv_pages(self):
        """(page_size, n_pages, n_free); page_size 0 for a contiguous cache."""
        ps, n, f = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        call("lmc_model_kv_pages", self.h, ctypes.byref(ps), ctypes.byref(n), ctypes.byref(f))
        return ps.value, n.value, f.value

    def replay(self, n):
        s = _vp()
        call("lmc_model_replay", self.h, n, ctypes.byref(s))
        return s.value

    def graph_kernels(self):
        return lib().lmc_model_graph_kernels(self.h)

    def close(self):
        if self.h:
            lib().lmc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def init(device=0):
    call("lmc_init", device)
