/*
 * strata_gguf.h — GGUF ingest for libstrata_cuda: a bounds-checked reader of
 * GGUF v3 model files (one file, or every shard of a split model) mapped
 * read-only, and the bulk upload of their tensors to HBM.
 *
 * The reader restates strata-gguf's (crates/strata-gguf/src/reader.rs):
 *   strata_cuda_gguf_open        GgufModel::open (:466-481) over split_paths (:527-572),
 *                                GgufFile::open/parse (:231-352) for each shard
 *   strata_cuda_gguf_tensor      TensorInfo (:179-199) with its shard, in shard then file order
 *   strata_cuda_gguf_find        GgufModel::find (:497-501)
 *   strata_cuda_gguf_tensor_data GgufModel::tensor_data (:504-507): GgufFile::tensor_data (:425-445)
 *                                over tensor_payload_bytes (:399-423)
 *   strata_cuda_gguf_meta        GgufModel::get (:492-494), MetaValue (metadata.rs:51-111)
 *   strata_cuda_gguf_split_paths split_paths (:527-572)
 * with the same checks and the same error for each failure: the status codes
 * below map one to one onto strata_gguf::Error (crates/strata-gguf/src/error.rs),
 * and the message carries that error's text.
 *
 * strata_cuda_gguf_ingest uploads a list of the model's tensors through
 * strata_cuda_upload_many, viewing each as strata-core's WeightStore does
 * (crates/strata-core/src/weights.rs:122-152): 1-D -> one row, 2-D
 * [cols, rows] -> a QuantTensor, 3-D [cols, rows, n_expert] -> an ExpertView.
 *
 * The reader needs no GPU; a model handle is read-only after open and may be
 * shared between threads. Payload pointers stay valid until the model is closed.
 */
#ifndef STRATA_GGUF_H
#define STRATA_GGUF_H

#include <stddef.h>
#include <stdint.h>

#include "strata_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes beyond strata_cuda.h's (STRATA_ERR_TRUNCATED and
 * STRATA_ERR_UNSUPPORTED_QUANT are shared with it). */
enum {
    STRATA_ERR_IO = 10,                  /* Error::Io: a shard cannot be opened, mapped or found */
    STRATA_ERR_BAD_MAGIC = 11,           /* Error::BadMagic */
    STRATA_ERR_UNSUPPORTED_VERSION = 12, /* Error::UnsupportedVersion (only v3 is read) */
    STRATA_ERR_BAD_VALUE_TYPE = 13,      /* Error::BadValueType (also nesting too deep, array too long) */
    STRATA_ERR_BAD_KEY_LENGTH = 14,      /* Error::BadKeyLength (any string over 65535 bytes) */
    STRATA_ERR_STRING_NOT_UTF8 = 15,     /* Error::StringNotUtf8 */
    STRATA_ERR_TENSOR_NOT_FOUND = 16,    /* Error::TensorNotFound (also a duplicate tensor name) */
    STRATA_ERR_WRONG_TENSOR_DIMS = 17    /* Error::WrongTensorDims */
};

typedef struct strata_gguf strata_gguf; /* an opened model: every shard, one name index */

/* Opens the model that `any_shard` belongs to: `<stem>-NNNNN-of-MMMMM.gguf`
 * opens shards 1..M, any other path opens that one file. On failure *out is
 * NULL and, when err is not NULL, err holds the message (truncated to
 * err_len bytes, NUL-terminated). */
int strata_cuda_gguf_open(const char *any_shard, strata_gguf **out, char *err, size_t err_len);
void strata_cuda_gguf_close(strata_gguf *g);

/* The shard paths split_paths resolves for `any_shard`, each ended by '\n',
 * written to buf (the status is STRATA_ERR_INVALID when buf_len is too small;
 * *needed then holds the size). A missing shard is STRATA_ERR_IO naming it. */
int strata_cuda_gguf_split_paths(const char *any_shard, char *buf, size_t buf_len, size_t *needed, char *err,
                                 size_t err_len);

typedef struct {
    const char *path;
    uint32_t version;
    uint64_t alignment;  /* general.alignment when it is a positive integer, else 32 */
    uint64_t data_start; /* first byte of the data section (clamped to the file size on a metadata-only shard) */
    uint64_t file_size;
    int64_t n_tensors;
    int64_t n_metadata; /* distinct keys */
} strata_gguf_shard;

int strata_cuda_gguf_n_shards(const strata_gguf *g);
int strata_cuda_gguf_shard(const strata_gguf *g, int shard, strata_gguf_shard *out);

typedef struct {
    const char *name;  /* NUL-terminated; a name may itself hold NUL bytes (valid UTF-8), so: */
    uint64_t name_len; /* its length in bytes */
    uint32_t type;     /* Strata ggml type id as stored (not validated until the payload is asked for) */
    int32_t n_dims;    /* 1..4 */
    uint64_t dims[4];  /* GGUF order: dims[0] varies fastest; unused entries are 0 */
    uint64_t offset;   /* from the shard's data start */
    int32_t shard;     /* 0-based */
} strata_gguf_tensor;

/* Tensors across all shards, in shard order then directory order. */
int64_t strata_cuda_gguf_tensor_count(const strata_gguf *g);
int strata_cuda_gguf_tensor(const strata_gguf *g, int64_t index, strata_gguf_tensor *out);
/* STRATA_OK with *index set, or STRATA_ERR_TENSOR_NOT_FOUND with *index = -1.
 * The name is taken up to its first NUL byte. */
int strata_cuda_gguf_find(const strata_gguf *g, const char *name, int64_t *index);

/* The tensor's payload in the mapping: exactly the bytes its shape and type
 * need, bounds-checked against its shard. */
int strata_cuda_gguf_tensor_data(const strata_gguf *g, int64_t index, const uint8_t **data, uint64_t *nbytes,
                                 char *err, size_t err_len);

/* One metadata value of the first (metadata) shard. Scalars as in
 * MetaValue: the 8- to 32-bit integers, bool and i64 in `i` (u64 in `u`, with
 * `i` = 0), f32 and f64 in `f`; strings in `str`/`str_len` (owned by the
 * model); arrays give their element type and full count only. */
enum {
    STRATA_GGUF_U8 = 0, STRATA_GGUF_I8 = 1, STRATA_GGUF_U16 = 2, STRATA_GGUF_I16 = 3, STRATA_GGUF_U32 = 4,
    STRATA_GGUF_I32 = 5, STRATA_GGUF_F32 = 6, STRATA_GGUF_BOOL = 7, STRATA_GGUF_STRING = 8,
    STRATA_GGUF_ARRAY = 9, STRATA_GGUF_U64 = 10, STRATA_GGUF_I64 = 11, STRATA_GGUF_F64 = 12
};
typedef struct {
    uint32_t type;
    int64_t i;
    uint64_t u;
    double f;
    const char *str;
    uint64_t str_len;
    uint32_t elem;
    uint64_t count;
} strata_gguf_value;
/* STRATA_OK, or STRATA_ERR_INVALID when the key is absent (the key is taken
 * up to its first NUL byte). */
int strata_cuda_gguf_meta(const strata_gguf *g, const char *key, strata_gguf_value *out);

/* The upload item (strata_cuda.h) for rows [first, first + count) of a 1-D or
 * 2-D tensor (1-D: one row) or experts [first, first + count) of a 3-D one;
 * count < 0 means to the end. `bytes` points into the mapping, so a rank of a
 * row-sharded projection or of an expert-parallel MoE reads only its own
 * slice of the file; pass the items to strata_cuda_upload_many. */
int strata_cuda_gguf_view(const strata_gguf *g, int64_t index, int64_t first, int64_t count, strata_upload *out,
                          char *err, size_t err_len);

/* Uploads n of the model's tensors (by index) to HBM in one staged pass, as
 * strata_cuda_upload_many: all or nothing, errors on the context. A tensor
 * of 4 dims is refused (no WeightStore view has 4). */
int strata_cuda_gguf_ingest(strata_ctx *ctx, const strata_gguf *g, const int64_t *tensors, int64_t n,
                            strata_weight **out);

/* One MoE layer of a GGUF model on the device, as strata-core's load_layer
 * (crates/strata-core/src/moe.rs:147-188) finds it: blk.<layer>.ffn_gate_inp.weight
 * (the router), ffn_gate_exps / ffn_up_exps / ffn_down_exps.weight and, when
 * with_shared, ffn_gate_shexp / ffn_up_shexp / ffn_down_shexp.weight and
 * ffn_gate_inp_shexp.weight. Only experts [expert_begin, expert_end) of the
 * expert tensors are read and uploaded (expert_end <= 0: to the last one;
 * n_expert is the expert tensors' count), together with the other tensors
 * in one staged pass (strata_cuda_upload_many); then the layer is created
 * (strata_cuda_moe_create) with n_ff = gate_exps' columns. weights_out (8
 * entries, in strata_moe_desc's order) receives the handles the layer uses
 * (NULL for the shared expert's when not loaded): free them after
 * strata_cuda_moe_destroy. A missing tensor is STRATA_ERR_TENSOR_NOT_FOUND
 * naming it (MissingTensor there); nothing stays resident on an error. */
int strata_cuda_gguf_moe_layer(strata_ctx *ctx, const strata_gguf *g, int64_t layer, int64_t top_k,
                               int64_t expert_begin, int64_t expert_end, int with_shared, strata_moe **out,
                               strata_weight **weights_out);

#ifdef __cplusplus
}
#endif

#endif /* STRATA_GGUF_H */
