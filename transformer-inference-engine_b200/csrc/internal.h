// internal.h -- structures shared by the host-side translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/kv_cache.h"
#include "../../include/safetensors.h"
#include "common.cuh"
#include "page_table.h"

// The cache: per layer a key pool and a value pool of `rows` fp32 rows of
// n_embd floats, all layers in one device allocation each. Pages of
// KV_CACHE_PAGE_ROWS rows; sequence s's logical page p is physical page
// page_table[s * pages_per_seq + p]. kv_cache_create builds a one-sequence
// cache whose pages are in order, so each layer is one contiguous block of
// `capacity` rows. A pool for many sequences holds n_pages assignable pages
// per layer plus one scratch page; `pages` hands them to sequences as their
// contexts grow (kv_pool_map) and takes them back (kv_pool_release).
struct kv_cache {
    int n_layer = 0, n_embd = 0, capacity = 0, length = 0;
    int n_seq = 1, pages_per_seq = 0;
    bool contiguous = true;   // kv_cache_create's one-sequence layout (whole-layer views exist)
    size_t rows = 0;    // physical rows per layer
    size_t bytes = 0;   // reported footprint
    float* k = nullptr;
    float* v = nullptr;
    int* d_page_table = nullptr;
    tie::PageTable pages;   // pools only
};

namespace tie {

// A pool for n_seq sequences of up to `capacity` positions each, over n_pages
// physical pages per layer (0: enough for every sequence's whole capacity).
// No page is assigned yet.
kv_status kv_pool_create(int n_layer, int n_embd, int n_seq, int capacity, int n_pages, kv_cache** out);
// Assigns pages so that sequences [0, n_seq) each cover positions [0, length),
// then brings the device table up to date on `st` (ordered before the kernels
// that follow on it). KV_ERR_CAPACITY when too few pages are free (the pages
// assigned so far stay assigned), KV_ERR_ARG for a bad range.
kv_status kv_pool_map(kv_cache* c, int n_seq, int length, cudaStream_t st);
// Returns sequence seq's pages to the pool.
kv_status kv_pool_release(kv_cache* c, int seq);

inline PagedKV layer_view(const kv_cache* c, int layer) {
    PagedKV v;
    v.k = c->k + (size_t)layer * c->rows * c->n_embd;
    v.v = c->v + (size_t)layer * c->rows * c->n_embd;
    v.page_table = c->d_page_table;
    v.pages_per_seq = c->pages_per_seq;
    v.n_embd = c->n_embd;
    return v;
}

// Copies n floats between any two of host/device memory and waits for it.
cudaError_t copy_any(void* dst, const void* src, size_t bytes);

cudaError_t launch_gemm_nn(const float* A, int lda, const float* B, int ldb, float* C, int ldc,
                           int M, int N, int K, cudaStream_t st);

// Bytes [offset, offset + n) of tensor t's data (safetensors.cpp).
st_status st_tensor_read_range(const st_file* f, const st_tensor* t, uint64_t offset, void* dst, size_t n);

}  // namespace tie
