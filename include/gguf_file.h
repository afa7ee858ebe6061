/*
 * gguf_file.h -- C ABI of the GGUF tensor-view loader in libgguf_onnx_ops.so.
 *
 * Maps an unmodified .gguf file (format v2 / v3, little-endian), parses its header, metadata and
 * tensor infos, and copies raw tensor bytes (whole tensors or row ranges of them) into device
 * memory, where the ops of gguf_ops.h consume them without repacking.  This is the host side of
 * the "execute directly against an unmodified .gguf file" flow of docs/GGUF_ONNX_Custom_Ops.md:5-7
 * (ONNX Runtime GenAI's gguf_initializers); the parse accepts and rejects what gguf-py 0.19.0's
 * GGUFReader does (gguf/gguf_reader.py:111-186 header and alignment, :289-316 fields and tensor
 * infos, :318-360 tensor sizes and duplicate names), on this layout:
 *
 *   u32 magic "GGUF" | u32 version | u64 n_tensors | u64 n_kv
 *   n_kv x (string key | u32 value type | value)            string = u64 length + bytes
 *   n_tensors x (string name | u32 n_dims | u64 dims[n_dims] | u32 ggml type | u64 offset)
 *   padding to general.alignment (default 32) | tensor data (offsets relative to its start)
 *
 * dims[0] is the innermost (contiguous) extent, as in ggml's ne[0].  Every function returns a
 * status code of gguf_ops.h (gguf_last_error() holds the message) unless documented otherwise.
 * A GgufFile may be read from several threads; uploads on one handle are serialised.
 */
#ifndef GGUF_FILE_H_
#define GGUF_FILE_H_

#include <stdint.h>

#include "gguf_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct GgufFile GgufFile;

/* GGUF metadata value types (gguf/constants.py GGUFValueType). */
enum {
  GGUF_VAL_UINT8 = 0, GGUF_VAL_INT8 = 1, GGUF_VAL_UINT16 = 2, GGUF_VAL_INT16 = 3, GGUF_VAL_UINT32 = 4,
  GGUF_VAL_INT32 = 5, GGUF_VAL_FLOAT32 = 6, GGUF_VAL_BOOL = 7, GGUF_VAL_STRING = 8, GGUF_VAL_ARRAY = 9,
  GGUF_VAL_UINT64 = 10, GGUF_VAL_INT64 = 11, GGUF_VAL_FLOAT64 = 12
};

typedef struct {
  const char* name;    /* NUL-terminated, owned by the handle */
  int32_t type;        /* ggml type id (GGUF_TYPE_* and the rest of ggml's numbering) */
  int32_t n_dims;      /* 1..4 */
  int64_t dims[4];     /* dims[0] innermost; unused entries are 1 */
  int64_t offset;      /* byte offset of the tensor data from the start of the file */
  int64_t nbytes;      /* (n_elements / block_elems) * block_bytes */
  int64_t block_elems; /* ggml block size of the type (1 for plain types) */
  int64_t block_bytes; /* bytes per block */
  int64_t row_bytes;   /* bytes of one dims[0] row: (dims[0] / block_elems) * block_bytes */
} GgufTensorInfo;

typedef struct {
  const char* key;    /* NUL-terminated, owned by the handle */
  int32_t type;       /* GGUF_VAL_* */
  int32_t elem_type;  /* element type when type == GGUF_VAL_ARRAY, else -1 */
  int64_t count;      /* 1 for a scalar; the byte length of a STRING; the element count of an ARRAY */
  const void* data;   /* inside the mapping: scalar bytes / string bytes / first array element */
  int64_t nbytes;     /* bytes of the value in the file (ARRAY: all elements, string headers included) */
} GgufKv;

/* One copy of gguf_file_upload: bytes [byte_offset, byte_offset + nbytes) of tensor `tensor`
 * (nbytes < 0: to the end of the tensor) to the device address dst. */
typedef struct {
  int64_t tensor;
  int64_t byte_offset;
  int64_t nbytes;
  void* dst;
} GgufUploadItem;

/* Opens and parses path.  Malformed files (bad magic, version other than 2 / 3, truncated
 * sections, non-power-of-two alignment, more than 4 dims, unknown types, ragged rows, data beyond
 * the end of the file, duplicate tensor names) fail with GGUF_ERR_INVALID_ARGUMENT; a file that
 * cannot be opened or mapped with GGUF_ERR_IO.  *out stays NULL on failure. */
GGUF_OPS_API int gguf_file_open(const char* path, GgufFile** out);

/* Releases the mapping and the staging buffers (waits for copies still reading them).  NULL is a no-op. */
GGUF_OPS_API void gguf_file_close(GgufFile* f);

/* Format version (2 or 3), data alignment, byte offset of the tensor data section, file size. */
GGUF_OPS_API int gguf_file_header(const GgufFile* f, int32_t* version, int64_t* alignment, int64_t* data_offset,
                                  int64_t* file_size);

/* Host address of the mapped file (read-only), or NULL for a NULL handle. */
GGUF_OPS_API const void* gguf_file_data(const GgufFile* f);

GGUF_OPS_API int64_t gguf_file_tensor_count(const GgufFile* f);
GGUF_OPS_API int gguf_file_tensor_info(const GgufFile* f, int64_t i, GgufTensorInfo* out);
/* Index of the tensor called name, or -1. */
GGUF_OPS_API int64_t gguf_file_find_tensor(const GgufFile* f, const char* name);

GGUF_OPS_API int64_t gguf_file_kv_count(const GgufFile* f);
GGUF_OPS_API int gguf_file_kv(const GgufFile* f, int64_t i, GgufKv* out);
/* Index of the metadata key, or -1. */
GGUF_OPS_API int64_t gguf_file_find_kv(const GgufFile* f, const char* key);

/* ggml block size and bytes per block of a type id; GGUF_ERR_INVALID_ARGUMENT for unknown ids. */
GGUF_OPS_API int gguf_type_size(int32_t type, int64_t* block_elems, int64_t* block_bytes);

/*
 * Copies n items to device memory.  The bytes go through pinned staging buffers owned by the
 * handle (4 x 32 MiB, allocated on the first call): host threads copy a chunk of the mapping
 * into a free buffer while earlier chunks are in flight on `stream`.  Returns once every copy
 * has completed (the staging buffers are free again); the device memory then holds the bytes.
 * Item ranges must lie inside their tensor; dst pointers must be device memory of the current
 * device.  Replaces the initializer injection of docs/GGUF_ONNX_Custom_Ops.md:5-7 for users
 * outside ONNX Runtime.
 */
GGUF_OPS_API int gguf_file_upload(GgufFile* f, const GgufUploadItem* items, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GGUF_FILE_H_ */
