"""The greedy head entry point that allocates nothing (tie_head_argmax_noalloc).

Some callers cannot allocate device memory: a serving framework whose caching
allocator already owns the GPU's memory, a plugin inside a runtime that forbids
allocations outside its own allocator, a latency-bound loop that cannot take
cudaMalloc's implicit synchronisation. This entry point keeps its scratch (the
per-block partial maxima) in a fixed array inside the library instead.

It is checked here, through the C ABI, on two calls in a row that reuse the
shared scratch: the logits against the float64 product x . w^T (within the fp32
summation bound the kernel tests use) and against the existing tiled matmul
entry point of gemm_impl_sm100a, the greedy ids against model_argmax over its
own logits, and a call without logits against the ids of the call with them.
This file is collected last so a failure here comes after every other test.
"""
import ctypes as C

import numpy as np
import pytest

import tie_b200

pytestmark = pytest.mark.gpu


def _call(L, x, w, rows, vocab, k, logits, nxt, stream):
    return L.tie_head_argmax_noalloc(x.data_ptr(), k, w.data_ptr(), k, rows, vocab, k,
                                     logits.data_ptr() if logits is not None else None, vocab,
                                     nxt.data_ptr(), stream)


def test_noalloc_head_matches_existing_entry_points():
    import torch
    L = tie_b200.library()
    K, V = 768, 50257
    rng = np.random.default_rng(2024)
    w_h = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    w = torch.from_numpy(w_h).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call, rows in enumerate((5, 16)):  # two calls in a row on the shared scratch
        x_h = rng.standard_normal((rows, K)).astype(np.float32)
        x = torch.from_numpy(x_h).cuda()
        logits = torch.empty((rows, V), dtype=torch.float32, device="cuda")
        nxt = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
        assert _call(L, x, w, rows, V, K, logits, nxt, stream) == 0
        torch.cuda.synchronize()
        got_logits, got_next = logits.cpu().numpy(), nxt.cpu().numpy()
        exact = x_h.astype(np.float64) @ w_h.astype(np.float64).T
        scale = np.abs(x_h).astype(np.float64) @ np.abs(w_h).astype(np.float64).T
        assert np.all(np.abs(got_logits - exact) <= K * 6e-8 * scale), call
        ref_logits = tie_b200.gemm_tiled_bt(x_h, w_h)          # existing entry point
        assert np.all(np.abs(got_logits - ref_logits) <= 2 * K * 6e-8 * scale), call
        own = np.array([tie_b200.argmax(r) for r in got_logits], np.int32)
        assert np.array_equal(got_next, own), (call, got_next, own)
        # the same rows without a logits buffer: the same greedy ids
        nxt2 = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
        assert _call(L, x, w, rows, V, K, None, nxt2, stream) == 0
        torch.cuda.synchronize()
        assert np.array_equal(nxt2.cpu().numpy(), got_next), call


def test_noalloc_head_refuses_sizes_beyond_its_scratch():
    import torch
    L = tie_b200.library()
    x = torch.zeros((17, 64), dtype=torch.float32, device="cuda")
    w = torch.zeros((8, 64), dtype=torch.float32, device="cuda")
    nxt = torch.zeros(17, dtype=torch.int32, device="cuda")
    cap = tie_b200.MODEL_STATUS.index("MODEL_ERR_CAPACITY")
    assert _call(L, x, w, 17, 8, 64, None, nxt, None) == cap
    assert L.tie_head_argmax_noalloc(x.data_ptr(), 64, w.data_ptr(), 64, 1, 65537, 64, None, 65537,
                                     nxt.data_ptr(), None) == cap
    arg = tie_b200.MODEL_STATUS.index("MODEL_ERR_ARG")
    assert L.tie_head_argmax_noalloc(x.data_ptr(), 64, w.data_ptr(), 64, 1, 8, 62, None, 8,
                                     nxt.data_ptr(), None) == arg
