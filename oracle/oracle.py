"""Python side of the CPU checkers. TEST INFRASTRUCTURE ONLY.

Two checkers live under oracle/:

* ``Oracle`` -- ctypes wrapper of liboracle.so, the C restatement of the
  reference forward pass (oracle/gpt2_oracle.c).  Weights are read from the
  safetensors file with numpy and handed to the C code as flat arrays.
* ``run_reference`` -- runs oracle/_ref/ref_gpt2, the reference's own C engine
  compiled unmodified (oracle/Makefile ``ref`` target), and parses its output.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module; the product library never calls into it.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_BIN = os.path.join(HERE, "_ref", "ref_gpt2")
REF_INVENTORY_BIN = os.path.join(HERE, "_ref", "st_inventory")


def build(reference_root: str | None = None) -> None:
    """Compiles liboracle.so, and the reference binaries when the reference
    source tree is present (its location: `reference_root`, else the
    TIE_REFERENCE_ROOT environment variable, else the Makefile's default):
    its CPU engine, and its C callers linked with the engine's library."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    ref = reference_root or os.environ.get("TIE_REFERENCE_ROOT")
    extra = [f"REF={ref}"] if ref else []
    subprocess.run(["make", "-s", "-C", HERE, "ref-if-present"] + extra, check=True)
    # the reference's own C callers linked with the engine (needs the engine built)
    engine = os.path.join(os.path.dirname(HERE), "transformer-inference-engine_b200", "lib", "libtie_b200.so")
    if os.path.isfile(engine):
        subprocess.run(["make", "-s", "-C", HERE, "callers-if-present"] + extra, check=True)


def reference_available() -> bool:
    return os.path.isfile(REF_BIN) and os.access(REF_BIN, os.X_OK)


# ------------------------------------------------------------ weight reading --

def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """name -> float32 array, read with the standard library and numpy."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n).decode("utf-8"))
        base = 8 + n
        out = {}
        for name, e in header.items():
            if name == "__metadata__":
                continue
            assert e["dtype"] == "F32", f"{name}: {e['dtype']}"
            b, end = e["data_offsets"]
            f.seek(base + b)
            out[name] = np.frombuffer(f.read(end - b), dtype="<f4").reshape(e["shape"]).copy()
    return out


def read_config(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


def canonical_names(n_layer: int) -> list[str]:
    names = ["wte.weight", "wpe.weight", "ln_f.weight", "ln_f.bias"]
    for l in range(n_layer):
        p = f"h.{l}."
        names += [p + s for s in ("ln_1.weight", "ln_1.bias", "attn.c_attn.weight",
                                  "attn.c_attn.bias", "attn.c_proj.weight", "attn.c_proj.bias",
                                  "ln_2.weight", "ln_2.bias", "mlp.c_fc.weight", "mlp.c_fc.bias",
                                  "mlp.c_proj.weight", "mlp.c_proj.bias")]
    return names


# ------------------------------------------------------------ the restatement --

class _Cfg(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_head", C.c_int), ("n_embd", C.c_int),
                ("n_ctx", C.c_int), ("vocab", C.c_int), ("eps", C.c_float)]


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB_PATH):
            build()
        lib = C.CDLL(LIB_PATH)
        fp = C.POINTER(C.c_float)
        ip = C.POINTER(C.c_int32)
        lib.orc_create.restype = C.c_void_p
        lib.orc_create.argtypes = [C.POINTER(_Cfg), C.POINTER(fp), C.c_int, C.c_int]
        lib.orc_free.argtypes = [C.c_void_p]
        lib.orc_prefill.argtypes = [C.c_void_p, ip, C.c_int, fp, fp, C.c_int]
        lib.orc_decode_cached.argtypes = [C.c_void_p, ip, C.c_int, fp]
        lib.orc_decode_nocache.argtypes = [C.c_void_p, ip, C.c_int, fp]
        lib.orc_greedy.argtypes = [C.c_void_p, ip, C.c_int, C.c_int, ip, fp, fp]
        lib.orc_kv_length.argtypes = [C.c_void_p]
        lib.orc_kv_set_length.argtypes = [C.c_void_p, C.c_int]
        lib.orc_gemm_naive.argtypes = [C.c_int] * 3 + [fp, C.c_int, fp, C.c_int, fp, C.c_int]
        lib.orc_gemm_naive_bt.argtypes = lib.orc_gemm_naive.argtypes
        lib.orc_layernorm_normalize.argtypes = [fp, C.c_int, C.c_float, fp]
        lib.orc_argmax.argtypes = [fp, C.c_size_t]
        lib.orc_argmax.restype = C.c_int32
        _lib = lib
    return _lib


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _ip(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


class Oracle:
    """The C restatement over one set of weights (held alive by this object)."""

    def __init__(self, weights: str, config: str, cproj_transposed: bool = False,
                 kv_capacity: int | None = None):
        lib = _load()
        cfg = read_config(config)
        self.n_layer, self.n_head = int(cfg["n_layer"]), int(cfg["n_head"])
        self.n_embd, self.n_ctx = int(cfg["n_embd"]), int(cfg["n_ctx"])
        self.vocab = int(cfg["vocab_size"])
        t = read_safetensors(weights)
        self._arrays = [np.ascontiguousarray(t[n], dtype=np.float32)
                        for n in canonical_names(self.n_layer)]
        ptrs = (C.POINTER(C.c_float) * len(self._arrays))(*[_fp(a) for a in self._arrays])
        c = _Cfg(self.n_layer, self.n_head, self.n_embd, self.n_ctx, self.vocab,
                 float(np.float32(cfg["layer_norm_epsilon"])))
        self._h = lib.orc_create(C.byref(c), ptrs, int(cproj_transposed),
                                 int(kv_capacity if kv_capacity is not None else self.n_ctx))
        if not self._h:
            raise MemoryError("orc_create failed")
        self.tensors = t

    def close(self):
        if getattr(self, "_h", None):
            _load().orc_free(self._h)
            self._h = None

    __del__ = close

    def prefill(self, ids, write_cache: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((len(ids), self.vocab), dtype=np.float32)
        rc = _load().orc_prefill(self._h, _ip(ids), len(ids), _fp(out),
                                 C.POINTER(C.c_float)(), int(write_cache))
        if rc:
            raise RuntimeError(f"orc_prefill rc={rc}")
        return out

    def decode_cached(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float32)
        rc = _load().orc_decode_cached(self._h, _ip(ids), len(ids), _fp(out))
        if rc:
            raise RuntimeError(f"orc_decode_cached rc={rc}")
        return out

    def decode_nocache(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float32)
        rc = _load().orc_decode_nocache(self._h, _ip(ids), len(ids), _fp(out))
        if rc:
            raise RuntimeError(f"orc_decode_nocache rc={rc}")
        return out

    def kv_set_length(self, n: int) -> None:
        rc = _load().orc_kv_set_length(self._h, int(n))
        if rc:
            raise RuntimeError(f"orc_kv_set_length rc={rc}")

    def greedy(self, prompt, n_new: int):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_new, dtype=np.int32)
        t1 = np.empty(n_new, dtype=np.float32)
        t2 = np.empty(n_new, dtype=np.float32)
        rc = _load().orc_greedy(self._h, _ip(prompt), len(prompt), n_new, _ip(out), _fp(t1), _fp(t2))
        if rc:
            raise RuntimeError(f"orc_greedy rc={rc}")
        return out, t1, t2


def gemm_naive(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.empty((M, N), np.float32)
    _load().orc_gemm_naive(M, N, K, _fp(A), K, _fp(B), N, _fp(Cm), N)
    return Cm


def gemm_naive_bt(A: np.ndarray, Bt: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    Bt = np.ascontiguousarray(Bt, np.float32)
    M, K = A.shape
    N = Bt.shape[0]
    Cm = np.empty((M, N), np.float32)
    _load().orc_gemm_naive_bt(M, N, K, _fp(A), K, _fp(Bt), K, _fp(Cm), N)
    return Cm


def layernorm_normalize(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    _load().orc_layernorm_normalize(_fp(x), x.size, float(eps), _fp(out))
    return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(_load().orc_argmax(_fp(v), v.size))


# ----------------------------------------------------------- the reference --

def run_reference(weights, inventory, config, prompts: np.ndarray, n_new: int,
                  prefill_logits: str = "none", step_logits: bool = False,
                  cproj_transposed: bool = False, first_seq: int = 0, n_seq: int | None = None,
                  nocache: bool = False, timeout: float | None = None, topk: int = 2,
                  prefill_topk: bool = False):
    """Runs oracle/_ref/ref_gpt2 on rows [first_seq, first_seq + n_seq) of prompts.
    Returns (list of per-sequence dicts, timing dict)."""
    if not reference_available():
        raise FileNotFoundError(REF_BIN)
    prompts = np.ascontiguousarray(prompts, dtype=np.int32)
    S, T = prompts.shape
    n_seq = S - first_seq if n_seq is None else n_seq
    with tempfile.TemporaryDirectory() as td:
        ids_path, out_path = os.path.join(td, "ids.bin"), os.path.join(td, "out.bin")
        prompts.tofile(ids_path)
        cmd = [REF_BIN, weights, inventory, config, ids_path, str(n_seq), str(T), str(n_new),
               out_path, "--first-seq", str(first_seq), "--prefill-logits", prefill_logits]
        if cproj_transposed:
            cmd += ["--cproj", "transposed"]
        if step_logits:
            cmd += ["--step-logits"]
        if nocache:
            cmd += ["--nocache"]
        cmd += ["--topk", str(topk)]
        if prefill_topk:
            cmd += ["--prefill-topk"]
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
        if p.returncode != 0:
            raise RuntimeError(f"ref_gpt2 failed ({p.returncode}): {p.stderr.strip()}")
        timing = json.loads(p.stdout.strip().splitlines()[-1])
        V = int(read_config(config)["vocab_size"])
        raw = np.fromfile(out_path, dtype=np.uint8)
    seqs, off = [], 0

    def take(n, dt):
        nonlocal off
        a = raw[off:off + 4 * n].view(dt).copy()
        off += 4 * n
        return a

    for _ in range(n_seq):
        d = {"ids": take(n_new, np.int32),
             "topk_ids": take(n_new * topk, np.int32).reshape(n_new, topk),
             "topk_vals": take(n_new * topk, np.float32).reshape(n_new, topk)}
        d["top1"] = d["topk_vals"][:, 0]
        if topk > 1:
            d["top2"] = d["topk_vals"][:, 1]
        if prefill_topk:
            d["prefill_topk_ids"] = take(T * topk, np.int32).reshape(T, topk)
            d["prefill_topk_vals"] = take(T * topk, np.float32).reshape(T, topk)
        if prefill_logits == "all":
            d["prefill_logits"] = take(T * V, np.float32).reshape(T, V)
        elif prefill_logits == "last":
            d["prefill_logits"] = take(V, np.float32).reshape(1, V)
        if step_logits and n_new > 1:
            d["step_logits"] = take((n_new - 1) * V, np.float32).reshape(n_new - 1, V)
        seqs.append(d)
    assert off == raw.size, (off, raw.size)
    return seqs, timing
