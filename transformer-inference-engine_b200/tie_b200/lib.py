"""ctypes binding of libtie_b200.so (see the package docstring)."""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO_ROOT = os.path.dirname(PKG_ROOT)
LIB_PATH = os.environ.get("TIE_B200_LIB", os.path.join(PKG_ROOT, "lib", "libtie_b200.so"))
INCLUDE_DIR = os.path.join(REPO_ROOT, "include")

MODEL_STATUS = ["MODEL_OK", "MODEL_ERR_OPEN", "MODEL_ERR_CONFIG", "MODEL_ERR_INVENTORY",
                "MODEL_ERR_WEIGHTS", "MODEL_ERR_SHAPE", "MODEL_ERR_DTYPE", "MODEL_ERR_RANGE",
                "MODEL_ERR_CAPACITY", "MODEL_ERR_NOMEM", "MODEL_ERR_ARG", "MODEL_ERR_DEVICE"]
KV_STATUS = ["KV_OK", "KV_ERR_ARG", "KV_ERR_CAPACITY", "KV_ERR_NOMEM"]
for _i, _n in enumerate(MODEL_STATUS + KV_STATUS):
    globals()[_n] = _i if _n in MODEL_STATUS else KV_STATUS.index(_n)
MODEL_PATH_NOCACHE, MODEL_PATH_CACHE = 0, 1
TIE_STEP_PERSISTENT, TIE_STEP_CHAINED, TIE_STEP_STREAM = 0, 1, 2
TIE_WEIGHTS_F32, TIE_WEIGHTS_BF16, TIE_WEIGHTS_INT8 = 0, 1, 2
MODEL_CPROJ_AS_STORED, MODEL_CPROJ_TRANSPOSED = 0, 1

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int32)
_vp = C.c_void_p


class ModelConfig(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_head", C.c_int), ("n_embd", C.c_int),
                ("n_ctx", C.c_int), ("vocab_size", C.c_int), ("head_dim", C.c_int),
                ("layer_norm_epsilon", C.c_float), ("activation_function", C.c_char * 32)]


class TensorRecord(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("stored_shape", C.c_char * 32),
                ("inventory_orientation", C.c_char * 48), ("transposed_at_load", C.c_int),
                ("reconciliation", C.c_char * 96)]


GemmFn = C.CFUNCTYPE(None, C.c_int, C.c_int, C.c_int, _fp, C.c_int, _fp, C.c_int, _fp, C.c_int)


class GemmImpl(C.Structure):
    _fields_ = [("name", C.c_char_p), ("mul", GemmFn), ("mul_bt", GemmFn)]


def header_symbols() -> list[str]:
    """Every function and exported object declared in include/*.h."""
    names = []
    for f in sorted(os.listdir(INCLUDE_DIR)):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE_DIR, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            if not text[m.start():m.end()].lstrip().startswith(("typedef", "return", "#")):
                names.append(m.group(1))
        names += re.findall(r"^extern\s+const\s+\w+\s+(\w+)\s*;", text, flags=re.M)
    return sorted(set(names))


EXPORTED_SYMBOLS = header_symbols() if os.path.isdir(INCLUDE_DIR) else []

_lib = None


def library():
    """Loads libtie_b200.so; raises (no fallback) when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.isfile(LIB_PATH):
        raise ImportError(f"libtie_b200.so not built ({LIB_PATH}); run tie_b200.build")
    L = C.CDLL(LIB_PATH)
    sig = {
        "model_load": (C.c_int, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_int, C.POINTER(_vp)]),
        "model_load_on_device": (C.c_int, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_int, C.c_int,
                                           C.POINTER(_vp)]),
        "model_free": (None, [_vp]),
        "model_config_of": (C.POINTER(ModelConfig), [_vp]),
        "model_cproj_reading_of": (C.c_int, [_vp]),
        "model_tensor_record_count": (C.c_size_t, [_vp]),
        "model_tensor_record_at": (C.POINTER(TensorRecord), [_vp, C.c_size_t]),
        "model_set_gemm": (None, [_vp, _vp]),
        "model_gemm_of": (C.POINTER(GemmImpl), [_vp]),
        "model_reserve": (C.c_int, [_vp, C.c_size_t]),
        "model_prefill": (C.c_int, [_vp, _ip, C.c_size_t, _fp, C.c_size_t]),
        "model_decode_step": (C.c_int, [_vp, _ip, C.c_size_t, _fp, C.c_size_t]),
        "model_set_decode_path": (None, [_vp, C.c_int]),
        "model_decode_path_of": (C.c_int, [_vp]),
        "model_kv_reserve": (C.c_int, [_vp, C.c_size_t]),
        "model_kv_footprint_bytes": (C.c_size_t, [_vp]),
        "model_kv_capacity": (C.c_int, [_vp]),
        "model_kv_length": (C.c_int, [_vp]),
        "model_kv_set_length": (C.c_int, [_vp, C.c_int]),
        "model_kv_cache_of": (_vp, [_vp]),
        "model_decode_step_cached": (C.c_int, [_vp, _ip, C.c_size_t, _fp, C.c_size_t]),
        "model_argmax": (C.c_int32, [_fp, C.c_size_t]),
        "model_token_embedding": (_vp, [_vp]),
        "model_head_weight": (_vp, [_vp]),
        "model_layernorm_normalize": (None, [_fp, C.c_int, C.c_float, _fp]),
        "tie_attention_prefill": (C.c_int, [_fp, C.c_int, C.c_int, C.c_int, _fp]),
        "model_collect_attn_stats": (None, [_vp, C.c_int]),
        "model_attn_rowsum_range": (None, [_vp, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                           C.POINTER(C.c_size_t)]),
        "model_strerror": (C.c_char_p, [C.c_int]),
        "model_device": (C.c_int, [_vp]),
        "model_stream": (_vp, [_vp]),
        "model_weight_device_bytes": (C.c_size_t, [_vp]),
        "model_kernel_launches": (C.c_uint64, [_vp]),
        "model_decode_step_greedy": (C.c_int, [_vp, _ip, C.c_size_t, _ip]),
        "model_batch_reserve": (C.c_int, [_vp, C.c_size_t, C.c_size_t]),
        "model_batch_reserve_pages": (C.c_int, [_vp, C.c_size_t, C.c_size_t, C.c_size_t]),
        "model_batch_release": (C.c_int, [_vp, C.c_size_t]),
        "model_batch_free_pages": (C.c_size_t, [_vp]),
        "model_prefill_batch": (C.c_int, [_vp, _ip, C.c_size_t, C.c_size_t, _fp, C.c_size_t, _ip]),
        "model_decode_step_batch": (C.c_int, [_vp, _ip, C.c_size_t, _fp, C.c_size_t, _ip]),
        "model_generate_greedy": (C.c_int, [_vp, _ip, C.c_size_t, C.c_size_t, C.c_size_t, _ip]),
        "model_generate_greedy_device": (C.c_int, [_vp, _vp, C.c_size_t, C.c_size_t, C.c_size_t, _vp]),
        "model_time_kernel": (C.c_int, [_vp, C.c_int, C.c_size_t, C.c_size_t, C.c_int, _fp]),
        "model_set_step_kernel": (C.c_int, [_vp, C.c_int]),
        "model_debug_wait_drill": (C.c_int, [_vp, C.c_uint64]),
        "model_stream_trace": (C.c_int, [_vp, C.c_size_t, C.c_size_t, _vp, C.c_size_t, _vp, _vp]),
        "model_set_weight_format": (C.c_int, [_vp, C.c_int]),
        "model_weight_format": (C.c_int, [_vp]),
        "model_step_trace": (C.c_int, [_vp, C.c_size_t, C.c_size_t, _vp, C.c_size_t,
                                       C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
        "tie_last_device_error": (C.c_char_p, []),
        "tie_head_argmax_noalloc": (C.c_int, [_vp, C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                              _vp, C.c_int, _vp, _vp]),
        "kv_cache_footprint_for": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
        "kv_cache_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
        "kv_cache_destroy": (None, [_vp]),
        "kv_cache_n_layer": (C.c_int, [_vp]),
        "kv_cache_n_embd": (C.c_int, [_vp]),
        "kv_cache_capacity": (C.c_int, [_vp]),
        "kv_cache_footprint_bytes": (C.c_size_t, [_vp]),
        "kv_cache_length": (C.c_int, [_vp]),
        "kv_cache_set_length": (C.c_int, [_vp, C.c_int]),
        "kv_cache_write": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
        "kv_cache_append": (C.c_int, [_vp, C.c_int, _vp, _vp]),
        "kv_cache_advance": (C.c_int, [_vp]),
        "kv_cache_keys": (_vp, [_vp, C.c_int]),
        "kv_cache_values": (_vp, [_vp, C.c_int]),
        "kv_cache_key_row": (_vp, [_vp, C.c_int, C.c_int]),
        "kv_cache_value_row": (_vp, [_vp, C.c_int, C.c_int]),
        "kv_strerror": (C.c_char_p, [C.c_int]),
        "kv_cache_copy_layer_to_host": (C.c_int, [_vp, C.c_int, C.c_int, _fp, C.c_int]),
        "gemm_naive": (None, [C.c_int, C.c_int, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp, C.c_int]),
        "gemm_naive_bt": (None, [C.c_int, C.c_int, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp, C.c_int]),
        "st_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
        "st_close": (None, [_vp]),
        "st_count": (C.c_size_t, [_vp]),
        "st_strerror": (C.c_char_p, [C.c_int]),
        "st_header_length": (C.c_uint64, [_vp]),
        "st_data_offset": (C.c_uint64, [_vp]),
        "st_file_size": (C.c_uint64, [_vp]),
        "st_metadata": (C.c_char_p, [_vp, C.c_char_p]),
        "st_has_metadata": (C.c_int, [_vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class ModelError(RuntimeError):
    def __init__(self, status: int, where: str = ""):
        self.status = status
        name = MODEL_STATUS[status] if 0 <= status < len(MODEL_STATUS) else str(status)
        msg = library().model_strerror(status).decode()
        detail = ""
        if name == "MODEL_ERR_DEVICE":
            detail = (library().tie_last_device_error() or b"").decode()
            detail = f" [{detail}]" if detail else ""
        super().__init__(f"{where}: {name} ({msg}){detail}")


def _chk(rc, where):
    if rc != 0:
        raise ModelError(rc, where)
    return rc


def _ids(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _ip_of(a: np.ndarray):
    return a.ctypes.data_as(_ip)


def _fp_of(a: np.ndarray):
    return a.ctypes.data_as(_fp)


class Model:
    """One loaded model (the reference's ``model *``)."""

    def __init__(self, weights, inventory, config, cproj: int = MODEL_CPROJ_AS_STORED,
                 device: int | None = None):
        L = library()
        h = _vp()
        if device is None:
            rc = L.model_load(weights.encode(), inventory.encode(), config.encode(), cproj, C.byref(h))
        else:
            rc = L.model_load_on_device(weights.encode(), inventory.encode(), config.encode(), cproj,
                                        device, C.byref(h))
        _chk(rc, "model_load")
        self.h = h.value
        c = L.model_config_of(self.h).contents
        self.n_layer, self.n_head, self.n_embd = c.n_layer, c.n_head, c.n_embd
        self.n_ctx, self.vocab, self.head_dim = c.n_ctx, c.vocab_size, c.head_dim
        self.eps = c.layer_norm_epsilon
        self.activation = c.activation_function.decode()

    @staticmethod
    def load_status(weights, inventory, config, cproj=MODEL_CPROJ_AS_STORED) -> int:
        """model_load's status without keeping the model."""
        L = library()
        h = _vp()
        rc = L.model_load(weights.encode(), inventory.encode(), config.encode(), cproj, C.byref(h))
        if rc == 0:
            L.model_free(h)
        return rc

    def close(self):
        if getattr(self, "h", None):
            library().model_free(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- the reference API ------------------------------------------------
    def prefill(self, ids, check=True):
        ids = _ids(ids)
        out = np.empty((max(len(ids), 1), self.vocab), dtype=np.float32)
        rc = library().model_prefill(self.h, _ip_of(ids), len(ids), _fp_of(out), len(ids) * self.vocab)
        if check:
            _chk(rc, "model_prefill")
            return out
        return rc, out

    def decode_step(self, ids, check=True):
        ids = _ids(ids)
        out = np.empty(self.vocab, dtype=np.float32)
        rc = library().model_decode_step(self.h, _ip_of(ids), len(ids), _fp_of(out), self.vocab)
        if check:
            _chk(rc, "model_decode_step")
            return out
        return rc, out

    def decode_step_cached(self, ids, check=True):
        ids = _ids(ids)
        out = np.empty(self.vocab, dtype=np.float32)
        rc = library().model_decode_step_cached(self.h, _ip_of(ids), len(ids), _fp_of(out), self.vocab)
        if check:
            _chk(rc, "model_decode_step_cached")
            return out
        return rc, out

    def decode_step_greedy(self, ids, check=True):
        ids = _ids(ids)
        nxt = np.zeros(1, dtype=np.int32)
        rc = library().model_decode_step_greedy(self.h, _ip_of(ids), len(ids), _ip_of(nxt))
        if check:
            _chk(rc, "model_decode_step_greedy")
            return int(nxt[0])
        return rc, int(nxt[0])

    def reserve(self, n):
        return library().model_reserve(self.h, n)

    def set_decode_path(self, p):
        library().model_set_decode_path(self.h, p)

    def set_weight_format(self, fmt):
        """TIE_WEIGHTS_F32 (default), TIE_WEIGHTS_BF16 or TIE_WEIGHTS_INT8."""
        _chk(library().model_set_weight_format(self.h, fmt), "model_set_weight_format")

    def weight_format(self):
        return library().model_weight_format(self.h)

    def set_step_kernel(self, kind):
        """TIE_STEP_CHAINED (default), TIE_STEP_STREAM (the same arithmetic in five
        kernels per layer, weights streamed through shared memory) or
        TIE_STEP_PERSISTENT (decode steps of <= 4 sequences)."""
        _chk(library().model_set_step_kernel(self.h, kind), "model_set_step_kernel")

    def debug_wait_drill(self, limit_ns: int):
        """The next TIE_STEP_STREAM decode step waits on a barrier nothing completes
        for limit_ns and reports MODEL_ERR_DEVICE (model_debug_wait_drill)."""
        _chk(library().model_debug_wait_drill(self.h, int(limit_ns)), "model_debug_wait_drill")

    def stream_trace(self, rows: int, context: int) -> np.ndarray:
        """Global-timer stamps (ns) of one chained decode step's streaming
        matmuls: [kernel][cta][event] (model_stream_trace)."""
        per, n = C.c_size_t(), C.c_size_t()
        library().model_stream_trace(self.h, rows, context, None, 0, C.byref(per), C.byref(n))
        out = np.zeros((n.value, per.value), dtype=np.uint64)
        _chk(library().model_stream_trace(self.h, rows, context, out.ctypes.data_as(_vp), out.size,
                                          C.byref(per), C.byref(n)), "model_stream_trace")
        return out.reshape(n.value, -1, 8)

    def step_trace(self, rows: int, context: int) -> np.ndarray:
        """Global-timer stamps (ns) of one persistent decode step: [n_cta, per_cta]."""
        per, n = C.c_size_t(), C.c_size_t()
        library().model_step_trace(self.h, rows, context, None, 0, C.byref(per), C.byref(n))
        out = np.zeros((n.value, per.value), dtype=np.uint64)
        _chk(library().model_step_trace(self.h, rows, context, out.ctypes.data_as(_vp), out.size,
                                        C.byref(per), C.byref(n)), "model_step_trace")
        return out

    def decode_path(self):
        return library().model_decode_path_of(self.h)

    def kv_reserve(self, cap):
        return library().model_kv_reserve(self.h, cap)

    def kv_footprint(self):
        return library().model_kv_footprint_bytes(self.h)

    def kv_capacity(self):
        return library().model_kv_capacity(self.h)

    def kv_length(self):
        return library().model_kv_length(self.h)

    def kv_set_length(self, n):
        return library().model_kv_set_length(self.h, n)

    def kv_cache(self):
        return library().model_kv_cache_of(self.h)

    def kv_layer_to_host(self, layer, which, n_rows):
        out = np.empty((n_rows, self.n_embd), dtype=np.float32)
        rc = library().kv_cache_copy_layer_to_host(self.kv_cache(), layer, which, _fp_of(out), n_rows)
        if rc != 0:
            raise RuntimeError(f"kv_cache_copy_layer_to_host: {KV_STATUS[rc]}")
        return out

    def token_embedding_ptr(self):
        return library().model_token_embedding(self.h)

    def head_weight_ptr(self):
        return library().model_head_weight(self.h)

    def records(self):
        L = library()
        out = []
        for i in range(L.model_tensor_record_count(self.h)):
            r = L.model_tensor_record_at(self.h, i).contents
            out.append(dict(name=r.name.decode(), stored_shape=r.stored_shape.decode(),
                            inventory_orientation=r.inventory_orientation.decode(),
                            transposed_at_load=r.transposed_at_load,
                            reconciliation=r.reconciliation.decode()))
        return out

    def gemm_name(self):
        return library().model_gemm_of(self.h).contents.name.decode()

    def collect_attn_stats(self, on):
        library().model_collect_attn_stats(self.h, int(on))

    def attn_rowsum_range(self):
        lo, hi, rows = C.c_double(), C.c_double(), C.c_size_t()
        library().model_attn_rowsum_range(self.h, C.byref(lo), C.byref(hi), C.byref(rows))
        return lo.value, hi.value, rows.value

    # ---- additive API -------------------------------------------------------
    @property
    def stream(self) -> int:
        return library().model_stream(self.h) or 0

    @property
    def device(self) -> int:
        return library().model_device(self.h)

    def weight_bytes(self):
        return library().model_weight_device_bytes(self.h)

    def kernel_launches(self):
        return library().model_kernel_launches(self.h)

    def batch_reserve(self, n_seq, capacity):
        return _chk(library().model_batch_reserve(self.h, n_seq, capacity), "model_batch_reserve")

    def batch_reserve_pages(self, n_seq, capacity, n_pages):
        """A batch pool over n_pages physical KV pages, assigned as contexts grow."""
        return _chk(library().model_batch_reserve_pages(self.h, n_seq, capacity, n_pages),
                    "model_batch_reserve_pages")

    def batch_release(self, seq):
        return _chk(library().model_batch_release(self.h, seq), "model_batch_release")

    def batch_free_pages(self) -> int:
        return library().model_batch_free_pages(self.h)

    def prefill_batch(self, ids, want_logits=False, check=True):
        ids = _ids(ids)
        S, T = ids.shape
        nxt = np.zeros(S, dtype=np.int32)
        logits = np.empty((S, T, self.vocab), dtype=np.float32) if want_logits else None
        rc = library().model_prefill_batch(self.h, _ip_of(ids), S, T,
                                           _fp_of(logits) if want_logits else None,
                                           logits.size if want_logits else 0, _ip_of(nxt))
        if check:
            _chk(rc, "model_prefill_batch")
            return nxt, logits
        return rc, nxt, logits

    def decode_step_batch(self, ids, want_logits=False, check=True):
        ids = _ids(ids)
        S = len(ids)
        nxt = np.zeros(S, dtype=np.int32)
        logits = np.empty((S, self.vocab), dtype=np.float32) if want_logits else None
        rc = library().model_decode_step_batch(self.h, _ip_of(ids), S,
                                               _fp_of(logits) if want_logits else None,
                                               logits.size if want_logits else 0, _ip_of(nxt))
        if check:
            _chk(rc, "model_decode_step_batch")
            return nxt, logits
        return rc, nxt, logits

    def generate_greedy(self, prompts, n_new, check=True):
        prompts = _ids(prompts)
        S, T = prompts.shape
        out = np.zeros((S, n_new), dtype=np.int32)
        rc = library().model_generate_greedy(self.h, _ip_of(prompts), S, T, n_new, _ip_of(out))
        if check:
            _chk(rc, "model_generate_greedy")
            return out
        return rc, out

    KERNELS = {"decode_attention": 0, "decode_qkv": 1, "decode_fc": 2, "decode_mlp_proj": 3,
               "decode_head": 4, "prefill_attention": 5, "prefill_fc": 6, "decode_step": 7}

    def time_kernel(self, name: str, rows: int, context: int, iters: int = 20) -> float:
        """Average milliseconds per launch of one kernel, alone (model_time_kernel)."""
        ms = C.c_float()
        _chk(library().model_time_kernel(self.h, self.KERNELS[name], rows, context, iters, C.byref(ms)),
             "model_time_kernel")
        return ms.value

    def generate_greedy_device(self, d_prompts: int, n_seq, n_prompt, n_new, d_out: int):
        return _chk(library().model_generate_greedy_device(self.h, d_prompts, n_seq, n_prompt, n_new, d_out),
                    "model_generate_greedy_device")


def kv_footprint_for(n_layer, n_embd, capacity):
    return library().kv_cache_footprint_for(n_layer, n_embd, capacity)


def _gemm(fn, A, B, bt):
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[0] if bt else B.shape[1]
    Cm = np.empty((M, N), np.float32)
    fn(M, N, K, A.ctypes.data, K, B.ctypes.data, B.shape[1], Cm.ctypes.data, N)
    return Cm


def gemm_naive(A, B):
    return _gemm(library().gemm_naive, A, B, False)


def gemm_naive_bt(A, Bt):
    return _gemm(library().gemm_naive_bt, A, Bt, True)


def _impl():
    return GemmImpl.in_dll(library(), "gemm_impl_sm100a")


def gemm_tiled(A, B):
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.empty((M, N), np.float32)
    _impl().mul(M, N, K, _fp_of(A), K, _fp_of(B), N, _fp_of(Cm), N)
    return Cm


def gemm_tiled_bt(A, Bt):
    A = np.ascontiguousarray(A, np.float32)
    Bt = np.ascontiguousarray(Bt, np.float32)
    M, K = A.shape
    N = Bt.shape[0]
    Cm = np.empty((M, N), np.float32)
    _impl().mul_bt(M, N, K, _fp_of(A), K, _fp_of(Bt), K, _fp_of(Cm), N)
    return Cm


def attention_prefill(qkv, n_head):
    """The engine's causal prefill attention over host qkv [n_seq, T, 3 * n_head * 64]
    (fp32): returns [n_seq, T, n_head * 64]."""
    qkv = np.ascontiguousarray(qkv, dtype=np.float32)
    n_seq, T, w = qkv.shape
    if w != 3 * n_head * 64:
        raise ValueError("qkv rows must be 3 * n_head * 64 wide")
    out = np.empty((n_seq, T, n_head * 64), np.float32)
    rc = library().tie_attention_prefill(_fp_of(qkv), n_seq, T, n_head, _fp_of(out))
    if rc != 0:
        raise RuntimeError(f"tie_attention_prefill: status {rc} "
                           f"({(library().tie_last_device_error() or b'').decode()})")
    return out


def layernorm_normalize(x, eps):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    library().model_layernorm_normalize(_fp_of(x), x.size, eps, _fp_of(out))
    return out


def argmax(v):
    v = np.ascontiguousarray(v, np.float32)
    return int(library().model_argmax(_fp_of(v), v.size))
