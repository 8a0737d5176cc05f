/*
 * cfi_gguf.h -- read-only GGUF (v2 / v3) model files for libcfi_b200.so.
 *
 * The reference reads real Q8_0 / Q4_K_M weights through Ollama and gguf-py
 * (cuda-for-intel scripts/divergence/analyze_divergence.py:28-60); this is the same access in C:
 * the file is mapped read-only, the header, metadata and tensor table are parsed and checked
 * (every tensor inside the file, offsets aligned to general.alignment), and tensor data is handed
 * out as pointers into the mapping, in ggml's own block layout, ready to copy to the device.
 * Host-only: no CUDA call is made.  Errors are return codes (0 = success) with a message.
 */
#ifndef CFI_GGUF_H
#define CFI_GGUF_H
#include <stddef.h>
#include <stdint.h>

#ifndef CFI_API
#define CFI_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cfi_gguf cfi_gguf;

/* metadata value types (GGUF spec) */
enum {
    CFI_GGUF_U8 = 0, CFI_GGUF_I8 = 1, CFI_GGUF_U16 = 2, CFI_GGUF_I16 = 3, CFI_GGUF_U32 = 4, CFI_GGUF_I32 = 5,
    CFI_GGUF_F32 = 6, CFI_GGUF_BOOL = 7, CFI_GGUF_STRING = 8, CFI_GGUF_ARRAY = 9, CFI_GGUF_U64 = 10,
    CFI_GGUF_I64 = 11, CFI_GGUF_F64 = 12
};

/* Opens and validates `path`.  Returns 0 and *out, or -1 with a reason in why. */
CFI_API int cfi_gguf_open(const char *path, cfi_gguf **out, char *why, size_t why_len);
CFI_API void cfi_gguf_close(cfi_gguf *f);

CFI_API uint32_t cfi_gguf_version(const cfi_gguf *f);
CFI_API uint64_t cfi_gguf_alignment(const cfi_gguf *f);
CFI_API uint64_t cfi_gguf_data_offset(const cfi_gguf *f);

/* ---- metadata ---- */
CFI_API int64_t cfi_gguf_kv_count(const cfi_gguf *f);
CFI_API int64_t cfi_gguf_find_key(const cfi_gguf *f, const char *key); /* index or -1 */
CFI_API const char *cfi_gguf_key(const cfi_gguf *f, int64_t i);
/* value type; for arrays also the element type and count */
CFI_API int cfi_gguf_kv_type(const cfi_gguf *f, int64_t i, int *elem_type, uint64_t *count);
/* scalar numeric (and bool) values; array element `j` when the value is an array of numbers */
CFI_API int cfi_gguf_get_i64(const cfi_gguf *f, int64_t i, uint64_t j, int64_t *out);
CFI_API int cfi_gguf_get_f64(const cfi_gguf *f, int64_t i, uint64_t j, double *out);
/* string value (or element j of an array of strings): pointer into the mapping, not terminated */
CFI_API int cfi_gguf_get_str(const cfi_gguf *f, int64_t i, uint64_t j, const char **s, uint64_t *len);

/* ---- tensors ---- */
CFI_API int64_t cfi_gguf_tensor_count(const cfi_gguf *f);
CFI_API int64_t cfi_gguf_find_tensor(const cfi_gguf *f, const char *name); /* index or -1 */
/* name (NUL-terminated copy owned by f), ggml type, dims (ne[0] innermost; up to 4), byte size
 * (0 for a type whose block size is unknown) and a pointer to the data in the mapping */
CFI_API int cfi_gguf_tensor_info(const cfi_gguf *f, int64_t i, const char **name, uint32_t *ggml_type,
                                 uint32_t *n_dims, uint64_t dims[4], uint64_t *nbytes, const void **data);
/* bytes of `n` values of a ggml type (0 when unknown or n is not a whole number of blocks) */
CFI_API uint64_t cfi_gguf_type_bytes(uint32_t ggml_type, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif
