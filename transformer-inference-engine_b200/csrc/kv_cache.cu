// kv_cache.cu -- the key/value store in device memory (include/kv_cache.h).
//
// Storage and refusal rules follow the reference (src/kv_cache.c:150-271): the
// footprint is computed from the arguments, the buffers are zero-filled at
// creation, a write at or beyond capacity stores nothing, one length counter
// serves all layers, and every entry point tolerates NULL.
#include "internal.h"

#include <cstring>
#include <new>

namespace tie {

cudaError_t copy_any(void* dst, const void* src, size_t bytes) {
    if (!bytes) return cudaSuccess;
    cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyDefault);
    if (e != cudaSuccess) return e;
    return cudaDeviceSynchronize();
}

static kv_status create_impl(int n_layer, int n_embd, int n_seq, int capacity, bool contiguous, int n_pages,
                             kv_cache** out) {
    if (!out) return KV_ERR_ARG;
    *out = nullptr;
    if (n_layer <= 0 || n_embd <= 0 || capacity <= 0 || n_seq <= 0 || n_pages < 0) return KV_ERR_ARG;
    kv_cache* c = new (std::nothrow) kv_cache();
    if (!c) return KV_ERR_NOMEM;
    c->n_layer = n_layer;
    c->n_embd = n_embd;
    c->capacity = capacity;
    c->n_seq = n_seq;
    c->contiguous = contiguous;
    c->pages_per_seq = (capacity + KV_CACHE_PAGE_ROWS - 1) / KV_CACHE_PAGE_ROWS;
    // One sequence: exactly `capacity` rows (the last page may be partial, and
    // no position reaches past capacity), pages in order. A pool: n_pages
    // assignable pages plus the scratch page unmapped entries point at.
    if (!contiguous && n_pages == 0) n_pages = n_seq * c->pages_per_seq;
    c->rows = contiguous ? (size_t)capacity : (size_t)(n_pages + 1) * KV_CACHE_PAGE_ROWS;
    c->bytes = (size_t)n_layer * 2u * c->rows * (size_t)n_embd * sizeof(float);
    const size_t per = (size_t)n_layer * c->rows * n_embd * sizeof(float);
    const size_t entries = (size_t)n_seq * c->pages_per_seq;
    std::vector<int> table(entries);
    if (contiguous) {
        for (size_t i = 0; i < entries; ++i) table[i] = (int)i;   // pages in order
    } else {
        c->pages = tie::PageTable(n_seq, capacity, n_pages);
        table = c->pages.device_view();                          // all entries on the scratch page
    }
    // A one-sequence cache is managed memory: its kv_cache_keys/values/*_row
    // addresses are usable on the host too (the reference's callers read rows
    // through them between calls), and its pages live in device memory while
    // the kernels use them. A pool stays plain device memory.
    auto alloc = [&](float** p) {
        return contiguous ? cudaMallocManaged(p, per, cudaMemAttachGlobal) : cudaMalloc(p, per);
    };
    if (alloc(&c->k) != cudaSuccess || alloc(&c->v) != cudaSuccess ||
        cudaMalloc(&c->d_page_table, entries * sizeof(int)) != cudaSuccess ||
        cudaMemset(c->k, 0, per) != cudaSuccess || cudaMemset(c->v, 0, per) != cudaSuccess ||
        cudaMemcpy(c->d_page_table, table.data(), entries * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        kv_cache_destroy(c);
        return KV_ERR_NOMEM;
    }
    *out = c;
    return KV_OK;
}

kv_status kv_pool_create(int n_layer, int n_embd, int n_seq, int capacity, int n_pages, kv_cache** out) {
    return create_impl(n_layer, n_embd, n_seq, capacity, false, n_pages, out);
}

kv_status kv_pool_map(kv_cache* c, int n_seq, int length, cudaStream_t st) {
    if (!c || c->contiguous || n_seq < 0 || n_seq > c->n_seq || length < 0) return KV_ERR_ARG;
    if (length > c->capacity) return KV_ERR_CAPACITY;
    kv_status rc = KV_OK;
    for (int s = 0; s < n_seq; ++s)
        if (!c->pages.map(s, length)) {
            rc = KV_ERR_CAPACITY;
            break;
        }
    if (c->pages.dirty()) {
        // the host view is copied before the call returns (pageable source),
        // and the copy is ordered before every later kernel on `st`
        const std::vector<int>& view = c->pages.device_view();
        if (cudaMemcpyAsync(c->d_page_table, view.data(), view.size() * sizeof(int), cudaMemcpyHostToDevice, st) !=
            cudaSuccess) {
            cudaGetLastError();
            return KV_ERR_NOMEM;
        }
    }
    return rc;
}

kv_status kv_pool_release(kv_cache* c, int seq) {
    if (!c || c->contiguous || seq < 0 || seq >= c->n_seq) return KV_ERR_ARG;
    c->pages.release(seq);
    return KV_OK;
}

}  // namespace tie

extern "C" {

const char* kv_strerror(kv_status s) {
    switch (s) {
        case KV_OK: return "ok";
        case KV_ERR_ARG: return "a null pointer or a non-positive shape";
        case KV_ERR_CAPACITY: return "the position or length is at or beyond capacity";
        case KV_ERR_NOMEM: return "device allocation failed";
    }
    return "unknown";
}

size_t kv_cache_footprint_for(int n_layer, int n_embd, int capacity) {
    if (n_layer <= 0 || n_embd <= 0 || capacity <= 0) return 0;
    return (size_t)n_layer * 2u * (size_t)capacity * (size_t)n_embd * sizeof(float);
}

kv_status kv_cache_create(int n_layer, int n_embd, int capacity, kv_cache** out) {
    return tie::create_impl(n_layer, n_embd, 1, capacity, true, 0, out);
}

void kv_cache_destroy(kv_cache* c) {
    if (!c) return;
    cudaFree(c->k);
    cudaFree(c->v);
    cudaFree(c->d_page_table);
    delete c;
}

int kv_cache_n_layer(const kv_cache* c) { return c ? c->n_layer : 0; }
int kv_cache_n_embd(const kv_cache* c) { return c ? c->n_embd : 0; }
int kv_cache_capacity(const kv_cache* c) { return c ? c->capacity : 0; }
size_t kv_cache_footprint_bytes(const kv_cache* c) { return c ? c->bytes : 0u; }
int kv_cache_length(const kv_cache* c) { return c ? c->length : 0; }

kv_status kv_cache_set_length(kv_cache* c, int length) {
    if (!c || length < 0) return KV_ERR_ARG;
    if (length > c->capacity) return KV_ERR_CAPACITY;
    c->length = length;
    return KV_OK;
}

// Row `pos` of a one-sequence cache: its pages are in order, so the layer is
// one [capacity, n_embd] block. The row-level entry points serve only such
// caches; a multi-sequence pool has no single position axis and refuses them.
static size_t phys_row(const kv_cache* c, int pos) { return (size_t)pos; }

kv_status kv_cache_write(kv_cache* c, int layer, int pos, const float* k, const float* v) {
    if (!c || !k || !v || !c->contiguous) return KV_ERR_ARG;
    if (layer < 0 || layer >= c->n_layer) return KV_ERR_ARG;
    if (pos < 0) return KV_ERR_ARG;
    if (pos >= c->capacity) return KV_ERR_CAPACITY;  // checked before either store
    const size_t off = ((size_t)layer * c->rows + phys_row(c, pos)) * c->n_embd;
    const size_t n = (size_t)c->n_embd * sizeof(float);
    if (tie::copy_any(c->k + off, k, n) != cudaSuccess) { cudaGetLastError(); return KV_ERR_ARG; }
    if (tie::copy_any(c->v + off, v, n) != cudaSuccess) { cudaGetLastError(); return KV_ERR_ARG; }
    return KV_OK;
}

kv_status kv_cache_append(kv_cache* c, int layer, const float* k, const float* v) {
    if (!c) return KV_ERR_ARG;
    return kv_cache_write(c, layer, c->length, k, v);
}

kv_status kv_cache_advance(kv_cache* c) {
    if (!c) return KV_ERR_ARG;
    if (c->length >= c->capacity) return KV_ERR_CAPACITY;
    ++c->length;
    return KV_OK;
}

const float* kv_cache_keys(const kv_cache* c, int layer) {
    if (!c || !c->contiguous || layer < 0 || layer >= c->n_layer) return nullptr;
    return c->k + (size_t)layer * c->rows * c->n_embd;
}

const float* kv_cache_values(const kv_cache* c, int layer) {
    if (!c || !c->contiguous || layer < 0 || layer >= c->n_layer) return nullptr;
    return c->v + (size_t)layer * c->rows * c->n_embd;
}

const float* kv_cache_key_row(const kv_cache* c, int layer, int pos) {
    const float* base = kv_cache_keys(c, layer);
    if (!base || pos < 0 || pos >= c->capacity) return nullptr;
    return base + phys_row(c, pos) * c->n_embd;
}

const float* kv_cache_value_row(const kv_cache* c, int layer, int pos) {
    const float* base = kv_cache_values(c, layer);
    if (!base || pos < 0 || pos >= c->capacity) return nullptr;
    return base + phys_row(c, pos) * c->n_embd;
}

kv_status kv_cache_copy_layer_to_host(const kv_cache* c, int layer, int which, float* dst,
                                      int n_rows) {
    if (!c || !dst || !c->contiguous || layer < 0 || layer >= c->n_layer || (which != 0 && which != 1) ||
        n_rows < 0)
        return KV_ERR_ARG;
    if (n_rows > c->capacity) return KV_ERR_CAPACITY;
    const float* base = which == 0 ? kv_cache_keys(c, layer) : kv_cache_values(c, layer);
    if (tie::copy_any(dst, base, (size_t)n_rows * c->n_embd * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return KV_ERR_ARG;
    }
    return KV_OK;
}

}  // extern "C"
