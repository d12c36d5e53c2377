/*
 * bml_gguf.h -- C ABI of the GGUF loader of libbmlattn.so: the file parsed
 * on the host (memory-mapped, zero-copy tensor views) and tensors copied to
 * device memory through pinned staging buffers.
 *
 * Reference interface replaced (paths inside the SugarFreeDoNoSo/bml
 * project):
 *   crates/parser/src/gguf.rs:239-292   GgufParser::open (header, metadata
 *                                        KV, tensor infos, data section
 *                                        aligned to 32 bytes)
 *   crates/parser/src/gguf.rs:294-364   header, metadata, tensor_infos,
 *                                        architecture, get_metadata,
 *                                        find_tensor, tensor_data
 *   crates/parser/src/gguf.rs:371-592   decode_header, decode_string,
 *                                        decode_metadata_kv / _value,
 *                                        decode_tensor_info
 *   crates/parser/src/mmap.rs:29-70     MmapFile (read-only mapping)
 * and, new on this side, the upload of tensors into device memory that
 * the reference does by dequantising into a host f32 pool
 * (gguf_compiler.rs:763-881).
 *
 * Conventions are those of bml_attn.h.  The handle owns the mapping and
 * every string and array it returns; they stay valid until bml_gguf_close.
 * Parsing follows the reference: magic 0x46554747, version <= 3, at least
 * 24 bytes, metadata value types 0-12 (arrays nest), tensor types as
 * GgufDataType::from_u32 (gguf.rs:77-108; an unknown id fails the open),
 * data section at the end of the tensor infos rounded up to 32 bytes
 * (general.alignment is not read, as in the reference).
 */
#ifndef BML_GGUF_H
#define BML_GGUF_H

#include "bml_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct bml_gguf bml_gguf;

/* GGUF metadata value types (gguf.rs:112-129). */
#define BML_GGUF_META_U8     0
#define BML_GGUF_META_I8     1
#define BML_GGUF_META_U16    2
#define BML_GGUF_META_I16    3
#define BML_GGUF_META_U32    4
#define BML_GGUF_META_I32    5
#define BML_GGUF_META_F32    6
#define BML_GGUF_META_BOOL   7
#define BML_GGUF_META_STRING 8
#define BML_GGUF_META_ARRAY  9
#define BML_GGUF_META_U64    10
#define BML_GGUF_META_I64    11
#define BML_GGUF_META_F64    12

typedef struct bml_gguf_header {
    uint32_t magic;
    uint32_t version;
    uint64_t tensor_count;
    uint64_t metadata_kv_count;
    uint64_t data_offset; /* start of the tensor data section in the file */
    uint64_t file_size;
} bml_gguf_header;

typedef struct bml_gguf_tensor {
    const char *name;       /* NUL-terminated (invalid UTF-8 kept as is) */
    uint64_t name_len;
    uint32_t n_dims;
    uint32_t type;          /* GGUF tensor type id */
    const uint64_t *dims;   /* n_dims entries */
    uint64_t offset;        /* relative to the data section */
    /* The reference's tensor_data(): present = 0 where it returns None;
     * otherwise the view starts at data_offset and holds view_len bytes
     * (the exact size for fixed-size types, up to the end of the file for
     * quantized ones, gguf.rs:339-364). */
    int32_t present;
    uint64_t data_offset;
    uint64_t view_len;
    /* Exact stored size from the type's block layout (0 where the library
     * does not know the type's layout); what bml_gguf_upload copies. */
    uint64_t nbytes;
} bml_gguf_tensor;

/* A metadata value.  Scalars: `u` (unsigned), `i` (signed), `f` (float
 * types, widened to double) as the type calls for, bool in `u`.  Strings:
 * `str` / `len` (bytes, not NUL-terminated).  Arrays: `elem_type` and
 * `len` (element count); read elements with a longer path. */
typedef struct bml_gguf_value {
    uint32_t type;
    uint32_t elem_type;
    uint64_t len;
    uint64_t u;
    int64_t i;
    double f;
    const char *str;
} bml_gguf_value;

/* GgufParser::open.  BML_E_INVALID with the reason in bml_last_error() for
 * a file the reference rejects; *out is set on success only. */
bml_status bml_gguf_open(const char *path, bml_gguf **out);
bml_status bml_gguf_close(bml_gguf *g);
bml_status bml_gguf_get_header(const bml_gguf *g, bml_gguf_header *out);

/* Tensor infos in file order; find gives the first of that name
 * (find_tensor), or *index = UINT64_MAX when there is none. */
bml_status bml_gguf_tensor_info(const bml_gguf *g, uint64_t index, bml_gguf_tensor *out);
bml_status bml_gguf_find_tensor(const bml_gguf *g, const char *name, uint64_t *index);
/* Zero-copy host view of tensor_data(): *ptr into the mapping, *len bytes;
 * *ptr = NULL where the reference returns None. */
bml_status bml_gguf_tensor_view(const bml_gguf *g, uint64_t index, const void **ptr, uint64_t *len);

/* Metadata entries in file order (metadata_kv_count of them).  find gives
 * the last entry with that key -- the one the reference's HashMap keeps --
 * or *index = UINT64_MAX.  A value is addressed by its entry and a path of
 * array indices (depth 0 for the entry's own value). */
bml_status bml_gguf_meta_key(const bml_gguf *g, uint64_t index, const char **key, uint64_t *key_len);
bml_status bml_gguf_meta_find(const bml_gguf *g, const char *key, uint64_t *index);
bml_status bml_gguf_meta_value(const bml_gguf *g, uint64_t index, const uint64_t *path, uint32_t depth,
                               bml_gguf_value *out);

/* Copies tensors into device memory: tensor indices[k]'s nbytes bytes to
 * dev_dst[k] (device pointers the caller allocated, on the current device).
 * The bytes go through pinned host staging buffers the handle allocates on
 * first use (one of 32 MiB per thread, freed by bml_gguf_close), filled by
 * `threads` host threads (0 = 8, at most 16) that each queue their copies
 * on their own stream.  Returns once every copy is done.
 * A tensor whose nbytes is 0 (unknown layout) or that runs past the end of
 * the file is refused before anything is copied. */
bml_status bml_gguf_upload(bml_gguf *g, const uint64_t *indices, uint32_t n, void *const *dev_dst,
                           uint32_t threads);

#ifdef __cplusplus
}
#endif

#endif /* BML_GGUF_H */
