"""tie_b200 -- Python binding of the B200 GPT-2 engine's C ABI.

The engine is ``lib/libtie_b200.so`` (built by ``tie_b200.build``); this package
only loads it with ctypes and mirrors the reference's C interface
(``include/model.h``, ``include/kv_cache.h``, ``include/gemm.h``) plus the
additive entry points of ``include/tie_b200.h``.  There is no Python or CPU
implementation of the forward pass here: importing the binding fails loudly when
the library is missing.
"""
from .lib import (  # noqa: F401
    LIB_PATH, MODEL_STATUS, KV_STATUS, ModelError, Model, library, kv_footprint_for,
    gemm_naive, gemm_naive_bt, gemm_tiled, gemm_tiled_bt, layernorm_normalize, attention_prefill, argmax,
    MODEL_PATH_NOCACHE, MODEL_PATH_CACHE, TIE_STEP_PERSISTENT, TIE_STEP_CHAINED, TIE_STEP_STREAM,
    TIE_WEIGHTS_F32, TIE_WEIGHTS_BF16, TIE_WEIGHTS_INT8, MODEL_CPROJ_AS_STORED, MODEL_CPROJ_TRANSPOSED,
    EXPORTED_SYMBOLS,
)
