/* safetensors.h -- weight-file reader used by model_load.
 *
 * Drop-in for the reference's src/safetensors.h (lines 47-117): same status and
 * dtype enums, same descriptor struct and the same st_* entry points, written
 * from the file format (an 8-byte little-endian header length, a JSON header of
 * {name: {dtype, shape, data_offsets}} plus an optional __metadata__ object,
 * then the unpadded data segment). Host-only; runs at load time.
 */
#ifndef TIE_B200_SAFETENSORS_H
#define TIE_B200_SAFETENSORS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ST_MAX_NAME  256
#define ST_MAX_DIMS  8

/* reference src/safetensors.h:50-65 */
typedef enum {
    ST_OK = 0,
    ST_ERR_OPEN,
    ST_ERR_READ,
    ST_ERR_TRUNCATED_HEADER,
    ST_ERR_BAD_JSON,
    ST_ERR_BAD_DTYPE,
    ST_ERR_BAD_SHAPE,
    ST_ERR_RANGE,
    ST_ERR_SIZE_MISMATCH,
    ST_ERR_NOT_FOUND,
    ST_ERR_TOO_MANY_DIMS,
    ST_ERR_NAME_TOO_LONG,
    ST_ERR_NOMEM,
    ST_ERR_ARG
} st_status;

/* reference src/safetensors.h:70-76 */
typedef enum {
    ST_DTYPE_UNKNOWN = 0,
    ST_DTYPE_BOOL, ST_DTYPE_U8, ST_DTYPE_I8,
    ST_DTYPE_U16, ST_DTYPE_I16, ST_DTYPE_F16, ST_DTYPE_BF16,
    ST_DTYPE_U32, ST_DTYPE_I32, ST_DTYPE_F32,
    ST_DTYPE_U64, ST_DTYPE_I64, ST_DTYPE_F64
} st_dtype;

/* reference src/safetensors.h:78-87 (identical layout) */
typedef struct {
    char     name[ST_MAX_NAME];
    st_dtype dtype;
    int      n_dims;
    int64_t  dims[ST_MAX_DIMS];
    uint64_t begin;
    uint64_t end;
    uint64_t file_offset;
    uint64_t nbytes;
} st_tensor;

typedef struct st_file st_file;

/* reference safetensors.h:93-117 */
st_status        st_open(const char *path, st_file **out);
void             st_close(st_file *f);
size_t           st_count(const st_file *f);
const st_tensor *st_at(const st_file *f, size_t index);
st_status        st_find(const st_file *f, const char *name, const st_tensor **out);
st_status        st_tensor_read(const st_file *f, const st_tensor *t, void *dst, size_t dst_bytes);
uint64_t         st_header_length(const st_file *f);
uint64_t         st_data_offset(const st_file *f);
uint64_t         st_file_size(const st_file *f);
const char      *st_metadata(const st_file *f, const char *key);
int              st_has_metadata(const st_file *f);
size_t           st_dtype_size(st_dtype d);
const char      *st_dtype_name(st_dtype d);
const char      *st_strerror(st_status s);

#ifdef __cplusplus
}
#endif

#endif /* TIE_B200_SAFETENSORS_H */
