"""Kernel-level parity on the GPU, through the C ABI (gemm.h and the LayerNorm
entry point).  The naive matmul performs the reference's exact float operations,
so it must match the CPU oracle BIT FOR BIT; the tiled kernels are compared with
a float64 product at a stated tolerance."""
import numpy as np
import pytest

import oracle
import tie_b200

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def lcg(n, seed):
    s, out = seed, np.empty(n, np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32((s >> 8) / 8388608.0 - 1.0)
    return out


def test_naive_hand_values():
    """reference tests/test_gemm_naive.c:71-93"""
    A = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    B = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    assert tie_b200.gemm_naive(A, B).tolist() == [[58, 64], [139, 154]]
    assert tie_b200.gemm_naive_bt(A, B.T.copy()).tolist() == [[58, 64], [139, 154]]


def test_naive_identity_exact():
    A = lcg(49, 12345).reshape(7, 7)
    I = np.eye(7, dtype=np.float32)
    assert np.array_equal(tie_b200.gemm_naive(A, I), A)
    assert np.array_equal(tie_b200.gemm_naive(I, A), A)
    assert np.array_equal(tie_b200.gemm_naive_bt(A, I), A)


@pytest.mark.parametrize("M,K,N", [(5, 3, 8), (8, 3, 5), (8, 768, 768), (3, 3072, 768)])
def test_naive_bit_exact_vs_oracle(M, K, N):
    rng = np.random.default_rng(M * 1000 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    assert np.array_equal(bits(tie_b200.gemm_naive(A, B)), bits(oracle.gemm_naive(A, B)))
    Bt = B.T.copy()
    assert np.array_equal(bits(tie_b200.gemm_naive_bt(A, Bt)), bits(oracle.gemm_naive_bt(A, Bt)))


def test_naive_leading_dimensions_and_untouched_columns():
    """reference tests/test_gemm_naive.c:146-167: a sub-block with ld > dims;
    nothing outside the N columns of C is written."""
    L = tie_b200.library()
    M, K, N, LDA, LDB, LDC = 4, 3, 2, 11, 9, 7
    A = lcg(M * LDA, 4242).reshape(M, LDA)
    B = lcg(K * LDB, 99).reshape(K, LDB)
    Cm = np.full((M, LDC), 12345.0, np.float32)
    L.gemm_naive(M, N, K, A.ctypes.data, LDA, B.ctypes.data, LDB, Cm.ctypes.data, LDC)
    ref = oracle.gemm_naive(np.ascontiguousarray(A[:, :K]), np.ascontiguousarray(B[:, :N]))
    assert np.array_equal(bits(Cm[:, :N]), bits(ref))
    assert np.all(Cm[:, N:] == 12345.0)


def test_naive_empty_sum_writes_zero():
    L = tie_b200.library()
    A = np.array([[3.0]], np.float32)
    Cm = np.array([[-1.0]], np.float32)
    L.gemm_naive(1, 1, 0, A.ctypes.data, 1, A.ctypes.data, 1, Cm.ctypes.data, 1)
    assert Cm[0, 0] == 0.0
    Cm[0, 0] = 5.0
    L.gemm_naive_bt(1, 1, 0, A.ctypes.data, 1, A.ctypes.data, 1, Cm.ctypes.data, 1)
    assert Cm[0, 0] == 0.0


@pytest.mark.parametrize("M,K,N", [(1, 768, 2304), (7, 768, 3072), (130, 3072, 768),
                                   (300, 768, 50257), (64, 1600, 4800), (9, 5, 3), (257, 1024, 4096)])
def test_tiled_bt_vs_float64(M, K, N):
    """The public mul_bt: the 3xTF32 tensor-core kernel when K % 32 == 0 (error
    bound K * 2^-20 * sum|a||b|, the split's per-product error summed
    coherently), else the fp32 FFMA kernel (K * 2^-24)."""
    rng = np.random.default_rng(M + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bt = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    got = tie_b200.gemm_tiled_bt(A, Bt)
    ref = A.astype(np.float64) @ Bt.astype(np.float64).T
    scale = np.abs(A).astype(np.float64) @ np.abs(Bt).astype(np.float64).T
    bound = K * (2.0 ** -20 if K % 32 == 0 else 6e-8)
    err = np.abs(got - ref)
    assert np.all(err <= bound * scale + 1e-30), float((err / scale).max())
    # typical error is fp32-level, far inside the bound
    assert np.median(err / scale) < 1e-6


def test_tiled_nn_and_batch_invariance():
    rng = np.random.default_rng(5)
    A = rng.standard_normal((200, 768)).astype(np.float32)
    B = (rng.standard_normal((768, 640)) * 0.02).astype(np.float32)
    full = tie_b200.gemm_tiled(A, B)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    assert np.abs(full - ref).max() < 1e-4
    # a row's result does not depend on the other rows of the batch (rows in
    # the first and second 128-row tile of the tensor-core kernel)
    Bt = B.T.copy()
    fullbt = tie_b200.gemm_tiled_bt(A, Bt)
    for r in (0, 77, 130, 199):
        one = tie_b200.gemm_tiled_bt(A[r:r + 1], Bt)
        assert np.array_equal(bits(one[0]), bits(fullbt[r]))


def test_layernorm_normalize_device():
    """reference tests/test_model.c:80-99 on the engine's LayerNorm kernel, and
    agreement with the oracle's sequential double statistics to one ulp."""
    x = lcg(768, 11) * np.float32(7.0) + np.float32(3.0)
    y = tie_b200.layernorm_normalize(x, 1e-5)
    yd = y.astype(np.float64)
    assert abs(yd.mean()) < 1e-5 and abs(yd.var() - 1.0) < 1e-4
    ref = oracle.layernorm_normalize(x, 1e-5)
    ulps = np.abs(bits(y).astype(np.int64) - bits(ref).astype(np.int64))
    assert ulps.max() <= 1


def attention_f64(qkv, n_head):
    """Causal attention in float64 (reference model.c:705-732: q.k / sqrt(64),
    mask, max-subtracted softmax, probability-weighted sum of v)."""
    n_seq, T, _ = qkv.shape
    E = n_head * 64
    q = qkv[..., :E].astype(np.float64).reshape(n_seq, T, n_head, 64)
    k = qkv[..., E:2 * E].astype(np.float64).reshape(n_seq, T, n_head, 64)
    v = qkv[..., 2 * E:].astype(np.float64).reshape(n_seq, T, n_head, 64)
    s = np.einsum("sqhd,skhd->shqk", q, k) / 8.0
    s = np.where(np.tril(np.ones((T, T), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.einsum("shqk,skhd->sqhd", p, v).reshape(n_seq, T, E)


@pytest.mark.parametrize("T", [1, 5, 63, 64, 65, 127, 128, 129, 300, 1024])
def test_prefill_attention_tensor_cores_vs_float64(T):
    """The tcgen05 prefill attention (3xTF32 products, 64-key blocks, 128-query
    tiles) against float64, on ragged and tile-aligned lengths."""
    n_seq, n_head = 2, 3
    qkv = np.random.default_rng(T).standard_normal((n_seq, T, 3 * n_head * 64)).astype(np.float32)
    got = tie_b200.attention_prefill(qkv, n_head)
    ref = attention_f64(qkv, n_head)
    err = np.abs(got - ref).max()
    assert err <= 2e-5, err


def test_prefill_attention_rows_do_not_depend_on_length():
    """Row t of a T-token prefill is bit-identical to row t of any longer one
    (causality; the key blocks past a row's diagonal add exact zeros)."""
    qkv = np.random.default_rng(7).standard_normal((1, 400, 3 * 64)).astype(np.float32)
    full = tie_b200.attention_prefill(qkv, 1)
    for t in (1, 64, 129, 255, 256, 399):
        part = tie_b200.attention_prefill(qkv[:, :t], 1)
        assert np.array_equal(bits(part), bits(full[:, :t])), t
