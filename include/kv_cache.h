/* kv_cache.h -- the per-layer key/value store, resident in B200 HBM.
 *
 * Drop-in for the reference's src/kv_cache.h (lines 41-102): same names, same
 * status codes, same refusal rules (a write at or beyond capacity is refused and
 * stores nothing; every entry point tolerates a NULL cache).
 *
 * Storage. Each layer has a key pool and a value pool of fp32 rows of n_embd
 * floats, with the heads contiguous along the row (the reference's activation
 * layout, kv_cache.h:10-18). Rows are grouped into pages of
 * KV_CACHE_PAGE_ROWS positions; attention kernels reach a position through a
 * page table, which is what lets the batch API (tie_b200.h) hand pages of one
 * pool to many sequences. A cache made by kv_cache_create belongs to one
 * sequence and maps its pages in order, so its layer buffer is one contiguous
 * [capacity, n_embd] block and the reference's addressing (row p at
 * base + p * n_embd) holds exactly.
 *
 * Pointers. For a cache made by kv_cache_create, kv_cache_keys/values/*_row
 * return addresses in CUDA managed memory: the kernels read them on the device,
 * and a caller may read rows through them on the host between calls (as the
 * reference's own tests and callers do; the first device access after a host
 * read migrates the touched pages back). Multi-sequence pools (the batch API)
 * are plain device memory: their whole-layer and row views are NULL and
 * kv_cache_write refuses them with KV_ERR_ARG. The store functions accept host
 * or device source rows (the copy direction is inferred from the pointer).
 * kv_cache_copy_layer_to_host reads a layer back into a host buffer.
 *
 * Footprint: n_layer * 2 * capacity * n_embd * 4 bytes, computed from the
 * arguments (reference kv_cache.h:20-22).
 */
#ifndef TIE_B200_KV_CACHE_H
#define TIE_B200_KV_CACHE_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Positions per page of a paged pool. */
#define KV_CACHE_PAGE_ROWS 16

/* reference src/kv_cache.h:41-46 */
typedef enum {
    KV_OK = 0,
    KV_ERR_ARG,        /* null pointer or non-positive shape           */
    KV_ERR_CAPACITY,   /* position or length at or beyond capacity     */
    KV_ERR_NOMEM       /* device allocation failed (or no device)      */
} kv_status;

typedef struct kv_cache kv_cache;

/* reference kv_cache.h:52. 0 for any non-positive argument. */
size_t kv_cache_footprint_for(int n_layer, int n_embd, int capacity);

/* reference kv_cache.h:56. Allocates device memory and zero-fills it here,
 * outside any timed region. */
kv_status kv_cache_create(int n_layer, int n_embd, int capacity, kv_cache **out);

/* reference kv_cache.h:59. NULL-safe. */
void kv_cache_destroy(kv_cache *c);

/* reference kv_cache.h:61-64 */
int    kv_cache_n_layer(const kv_cache *c);
int    kv_cache_n_embd(const kv_cache *c);
int    kv_cache_capacity(const kv_cache *c);
size_t kv_cache_footprint_bytes(const kv_cache *c);

/* reference kv_cache.h:72-73: one length counter for the whole cache. */
int       kv_cache_length(const kv_cache *c);
kv_status kv_cache_set_length(kv_cache *c, int length);

/* reference kv_cache.h:87-90. k and v are n_embd floats each, host or device. */
kv_status kv_cache_write(kv_cache *c, int layer, int pos, const float *k, const float *v);
kv_status kv_cache_append(kv_cache *c, int layer, const float *k, const float *v);
kv_status kv_cache_advance(kv_cache *c);

/* reference kv_cache.h:97-100. DEVICE pointers; NULL on a bad argument. */
const float *kv_cache_keys(const kv_cache *c, int layer);
const float *kv_cache_values(const kv_cache *c, int layer);
const float *kv_cache_key_row(const kv_cache *c, int layer, int pos);
const float *kv_cache_value_row(const kv_cache *c, int layer, int pos);

/* reference kv_cache.h:102 */
const char *kv_strerror(kv_status s);

/* Additive: copies rows [0, n_rows) of one layer's keys (which == 0) or values
 * (which == 1) into a host buffer of n_rows * n_embd floats. */
kv_status kv_cache_copy_layer_to_host(const kv_cache *c, int layer, int which,
                                      float *dst, int n_rows);

#ifdef __cplusplus
}
#endif

#endif /* TIE_B200_KV_CACHE_H */
