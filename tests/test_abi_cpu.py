"""The C ABI on the CPU: the library loads, exports every symbol include/*.h
declares, and behaves like the reference on every path that refuses or answers
before any device work (argument checks, artifact validation, pure arithmetic,
NULL tolerance).  No kernel is launched here."""
import ctypes as C
import json
import os
import shutil
import struct

import numpy as np
import pytest

import tie_b200
from tie_b200 import lib as tl

L = tie_b200.library()


def test_exports_every_declared_symbol():
    syms = tie_b200.EXPORTED_SYMBOLS
    assert len(syms) > 60
    missing = [s for s in syms if not hasattr(L, s)]
    assert missing == []


def test_header_declares_the_reference_api():
    """Every entry point of the reference's model.h / kv_cache.h / gemm.h /
    safetensors.h is declared (reference src/model.h:117-249, kv_cache.h:52-102,
    gemm/gemm.h:78-89, safetensors.h:93-117)."""
    ref_api = """model_load model_free model_config_of model_cproj_reading_of model_tensor_record_count
    model_tensor_record_at model_set_gemm model_gemm_of model_reserve model_prefill model_decode_step
    model_set_decode_path model_decode_path_of model_kv_reserve model_kv_footprint_bytes
    model_kv_capacity model_kv_length model_kv_set_length model_kv_cache_of model_decode_step_cached
    model_argmax model_token_embedding model_head_weight model_layernorm_normalize
    model_collect_attn_stats model_attn_rowsum_range model_strerror kv_cache_footprint_for
    kv_cache_create kv_cache_destroy kv_cache_n_layer kv_cache_n_embd kv_cache_capacity
    kv_cache_footprint_bytes kv_cache_length kv_cache_set_length kv_cache_write kv_cache_append
    kv_cache_advance kv_cache_keys kv_cache_values kv_cache_key_row kv_cache_value_row kv_strerror
    gemm_naive gemm_naive_bt gemm_impl_naive st_open st_close st_count st_at st_find st_tensor_read
    st_header_length st_data_offset st_file_size st_metadata st_has_metadata st_dtype_size
    st_dtype_name st_strerror""".split()
    assert sorted(set(ref_api) - set(tie_b200.EXPORTED_SYMBOLS)) == []


# ------------------------------------------------------------- kv_cache --

def test_kv_footprint_constants():
    """reference tests/test_kv_cache.c:40-60"""
    f = tie_b200.kv_footprint_for
    for cap in (1, 128, 1024):
        assert f(12, 768, cap) == 12 * 2 * cap * 768 * 4
    assert f(12, 768, 1024) == 75497472
    assert f(12, 768, 1) == 73728
    assert f(0, 768, 1024) == 0 and f(12, 0, 1024) == 0 and f(12, 768, 0) == 0


def test_kv_create_refuses_bad_shapes_without_allocating():
    """reference tests/test_kv_cache.c:77-90"""
    for args in ((0, 8, 4), (2, -1, 4), (2, 8, 0)):
        out = C.c_void_p(0xdeadbeef)
        assert L.kv_cache_create(*args, C.byref(out)) == tl.KV_STATUS.index("KV_ERR_ARG")
        assert out.value is None
    assert L.kv_cache_create(2, 8, 4, None) == tl.KV_STATUS.index("KV_ERR_ARG")
    L.kv_cache_destroy(None)


def test_kv_null_tolerance_and_strings():
    """reference tests/test_kv_cache.c:220-248"""
    arg = tl.KV_STATUS.index("KV_ERR_ARG")
    k = (C.c_float * 4)()
    assert L.kv_cache_write(None, 0, 0, k, k) == arg
    assert L.kv_cache_append(None, 0, k, k) == arg
    assert L.kv_cache_advance(None) == arg
    assert L.kv_cache_set_length(None, 0) == arg
    assert L.kv_cache_length(None) == 0 and L.kv_cache_capacity(None) == 0
    assert L.kv_cache_footprint_bytes(None) == 0 and L.kv_cache_keys(None, 0) is None
    strs = {L.kv_strerror(i) for i in range(4)}
    assert len(strs) == 4


# ---------------------------------------------------------------- model --

def test_model_strerror_distinct():
    s = [L.model_strerror(i) for i in range(len(tl.MODEL_STATUS))]
    assert len(set(s)) == len(s)
    assert b"CUDA" in L.model_strerror(tl.MODEL_STATUS.index("MODEL_ERR_DEVICE"))


def test_model_null_tolerance():
    assert not L.model_config_of(None)
    assert L.model_kv_length(None) == 0 and L.model_kv_capacity(None) == 0
    assert L.model_kv_footprint_bytes(None) == 0 and L.model_kv_cache_of(None) is None
    assert L.model_tensor_record_count(None) == 0
    assert L.model_decode_path_of(None) == tl.MODEL_PATH_NOCACHE
    L.model_free(None)
    arg = tl.MODEL_STATUS.index("MODEL_ERR_ARG")
    ids = (C.c_int32 * 2)(1, 2)
    out = (C.c_float * 8)()
    assert L.model_prefill(None, ids, 2, out, 8) == arg
    assert L.model_decode_step(None, ids, 2, out, 8) == arg
    assert L.model_decode_step_cached(None, ids, 2, out, 8) == arg
    assert L.model_kv_reserve(None, 4) == arg
    assert L.model_kv_set_length(None, 1) == arg


def test_model_argmax_host_rules():
    """reference src/model.c:920-925: strict '>' scan, lowest index on ties,
    a NaN never displaces the current best (so NaN at index 0 wins)."""
    a = tie_b200.argmax
    assert a(np.array([1, 3, 3, 2], np.float32)) == 1
    assert a(np.array([np.nan, 3, 4], np.float32)) == 0
    assert a(np.array([1, np.nan, 4, 4], np.float32)) == 2
    assert a(np.array([-np.inf, -np.inf], np.float32)) == 0


def _copy_artifacts(paths, tmp_path):
    w, inv, cfg = paths
    d = tmp_path / "m"
    d.mkdir()
    out = []
    for p in (w, inv, cfg):
        q = d / os.path.basename(p)
        shutil.copy(p, q)
        out.append(str(q))
    return out


def S(name):
    return tl.MODEL_STATUS.index(name)


def test_load_refusals_before_device(tiny_paths, tmp_path):
    """model_load refuses bad artifacts with the reference's status codes
    (src/model.c:337-467) before touching the GPU."""
    w, inv, cfg = _copy_artifacts(tiny_paths, tmp_path)
    load = tie_b200.Model.load_status
    assert load(w + ".missing", inv, cfg) == S("MODEL_ERR_WEIGHTS")
    assert load(w, inv + ".missing", cfg) == S("MODEL_ERR_OPEN")
    assert load(w, inv, cfg + ".missing") == S("MODEL_ERR_OPEN")

    base = json.load(open(cfg))

    def with_cfg(**kw):
        c = dict(base)
        for k, v in kw.items():
            if v is None:
                c.pop(k)
            else:
                c[k] = v
        json.dump(c, open(cfg, "w"))
        try:
            return load(w, inv, cfg)
        finally:
            json.dump(base, open(cfg, "w"))

    assert with_cfg(n_layer=None) == S("MODEL_ERR_CONFIG")
    assert with_cfg(layer_norm_epsilon=None) == S("MODEL_ERR_CONFIG")
    assert with_cfg(activation_function="gelu") == S("MODEL_ERR_CONFIG")
    assert with_cfg(n_head=3) == S("MODEL_ERR_CONFIG")            # 128 % 3 != 0
    assert with_cfg(n_head=4, n_embd=128) in (S("MODEL_ERR_CONFIG"), S("MODEL_ERR_INVENTORY"))
    assert with_cfg(n_layer=3) == S("MODEL_ERR_INVENTORY")       # inventory says 2
    # a real GPT-2 config carries booleans, nulls, floats and nested objects
    # beside the fields the loader reads; an unreadable or truncated text is refused
    raw = open(cfg).read()
    try:
        full = dict(base, scale_attn_weights=True, n_inner=None, resid_pdrop=0.1,
                    task_specific_params={"text-generation": {"do_sample": True, "max_length": 50}})
        json.dump(full, open(cfg, "w"), indent=2)
        assert load(w, inv, cfg) in (S("MODEL_OK"), S("MODEL_ERR_DEVICE"))
        open(cfg, "w").write(raw[: len(raw) // 2])
        assert load(w, inv, cfg) == S("MODEL_ERR_CONFIG")
        open(cfg, "w").write(raw.replace('"n_embd": 128', '"n_embd": "128"'))
        assert load(w, inv, cfg) == S("MODEL_ERR_CONFIG")
    finally:
        open(cfg, "w").write(raw)

    text = open(inv).read()

    def with_inv(new):
        open(inv, "w").write(new)
        try:
            return load(w, inv, cfg)
        finally:
            open(inv, "w").write(text)

    assert with_inv(text.replace('{"name": "h.1.ln_2.bias",', '{"name": "h.1.ln_2.biax",')) == \
        S("MODEL_ERR_INVENTORY")
    assert with_inv(text[: len(text) - 40]) == S("MODEL_ERR_INVENTORY")     # truncated
    line = [l for l in text.splitlines() if '"name": "h.0.mlp.c_fc.bias"' in l][0]
    assert with_inv(text.replace(line, line.replace('"F32"', '"F16"'))) == S("MODEL_ERR_DTYPE")
    assert with_inv(text.replace(line, line.replace('"shape": [512]', '"shape": [511]'))) == \
        S("MODEL_ERR_SHAPE")
    off = line.split('"file_offset": ')[1].split(",")[0]
    assert with_inv(text.replace(line, line.replace(f'"file_offset": {off}', f'"file_offset": {int(off) + 4}'))) \
        == S("MODEL_ERR_INVENTORY")
    assert L.model_load(None, inv.encode(), cfg.encode(), 0, C.byref(C.c_void_p())) == S("MODEL_ERR_ARG")


# ---------------------------------------------------------- safetensors --

def _st(tmp_path, header: bytes, data: bytes = b"", raw_len=None):
    p = tmp_path / "x.safetensors"
    n = len(header) if raw_len is None else raw_len
    p.write_bytes(struct.pack("<Q", n) + header + data)
    return str(p)


def _open(path):
    h = C.c_void_p()
    rc = L.st_open(path.encode(), C.byref(h))
    if rc == 0:
        L.st_close(h)
    return rc


ST = ["ST_OK", "ST_ERR_OPEN", "ST_ERR_READ", "ST_ERR_TRUNCATED_HEADER", "ST_ERR_BAD_JSON",
      "ST_ERR_BAD_DTYPE", "ST_ERR_BAD_SHAPE", "ST_ERR_RANGE", "ST_ERR_SIZE_MISMATCH",
      "ST_ERR_NOT_FOUND", "ST_ERR_TOO_MANY_DIMS", "ST_ERR_NAME_TOO_LONG", "ST_ERR_NOMEM", "ST_ERR_ARG"]


def test_safetensors_reader_facts(tiny_paths):
    w, _, _ = tiny_paths
    h = C.c_void_p()
    assert L.st_open(w.encode(), C.byref(h)) == 0
    n = struct.unpack("<Q", open(w, "rb").read(8))[0]
    assert L.st_header_length(h) == n and L.st_data_offset(h) == 8 + n
    assert L.st_file_size(h) == os.path.getsize(w)
    assert L.st_has_metadata(h) == 1 and L.st_metadata(h, b"format") == b"pt"
    assert L.st_count(h) == 4 + 12 * 2
    L.st_close(h)


def test_safetensors_reader_refusals(tmp_path):
    good = b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}'
    assert _open(_st(tmp_path, good, b"\0" * 8)) == 0
    assert _open(_st(tmp_path, good.replace(b"}}", b',"extra":[1,{"k":"v"}]}}'), b"\0" * 8)) == 0
    assert _open(_st(tmp_path, good, b"\0" * 8, raw_len=10 ** 6)) == ST.index("ST_ERR_TRUNCATED_HEADER")
    assert _open(_st(tmp_path, good[:-1], b"\0" * 8)) == ST.index("ST_ERR_BAD_JSON")
    assert _open(_st(tmp_path, good + b"x", b"\0" * 8)) == ST.index("ST_ERR_BAD_JSON")
    assert _open(_st(tmp_path, good.replace(b'"a"', b'"\\u0061"'), b"\0" * 8)) == ST.index("ST_ERR_BAD_JSON")
    assert _open(_st(tmp_path, good.replace(b"F32", b"F8"), b"\0" * 8)) == ST.index("ST_ERR_BAD_DTYPE")
    assert _open(_st(tmp_path, good.replace(b"[0,8]", b"[0,16]"), b"\0" * 8)) == ST.index("ST_ERR_RANGE")
    assert _open(_st(tmp_path, good.replace(b"[2]", b"[3]"), b"\0" * 8)) == ST.index("ST_ERR_SIZE_MISMATCH")
    assert _open(_st(tmp_path, good.replace(b"[2]", b"[-2]"), b"\0" * 8)) == ST.index("ST_ERR_BAD_SHAPE")
    assert _open(str(tmp_path / "nope")) == ST.index("ST_ERR_OPEN")


def test_gemm_zero_sized_writes_nothing():
    """reference tests/test_gemm_naive.c:190-206 (M or N zero: nothing written,
    no device work)."""
    A = np.ones((1, 1), np.float32)
    Cm = np.full((1, 1), 5.0, np.float32)
    L.gemm_naive(0, 1, 1, A.ctypes.data, 1, A.ctypes.data, 1, Cm.ctypes.data, 1)
    L.gemm_naive(1, 0, 1, A.ctypes.data, 1, A.ctypes.data, 1, Cm.ctypes.data, 1)
    assert Cm[0, 0] == 5.0
