/* Declaration-only stand-in for the ggml header, written for this repository so that the
 * reference's ggml-independent sources (scaler, refine, covariates, masks, and the F32
 * callbacks of layers/head) compile from their own files into the test oracle oracle/_ref.
 * Only the types and prototypes those sources name are declared; the graph-building
 * functions are defined in ref_shim.cpp (eager evaluation for custom nodes, abort for the
 * rest). This is test infrastructure, not the product. */
#pragma once
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_MAX_OP_PARAMS 64
#define GGML_MAX_NAME 64
#define GGML_TENSOR_FLAG_INPUT 1
enum ggml_type {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q4_1 = 3, GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7, GGML_TYPE_Q8_0 = 8, GGML_TYPE_Q8_1 = 9, GGML_TYPE_Q4_K = 12, GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14, GGML_TYPE_I32 = 26, GGML_TYPE_F64 = 28, GGML_TYPE_BF16 = 30
};
enum ggml_op { GGML_OP_NONE = 0, GGML_OP_CUSTOM = 1 };
enum ggml_status { GGML_STATUS_SUCCESS = 0 };
struct ggml_backend_buffer;
struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer* buffer;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    enum ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    struct ggml_tensor* src[GGML_MAX_SRC];
    void* data;
    char name[GGML_MAX_NAME];
};
struct ggml_context;
struct ggml_cgraph;
typedef void (*ggml_custom_op_t)(struct ggml_tensor* dst, int ith, int nth, void* userdata);

int64_t ggml_nelements(const struct ggml_tensor* t);
size_t ggml_nbytes(const struct ggml_tensor* t);
bool ggml_is_contiguous(const struct ggml_tensor* t);
bool ggml_are_same_shape(const struct ggml_tensor* a, const struct ggml_tensor* b);
int64_t ggml_blck_size(enum ggml_type type);
const char* ggml_type_name(enum ggml_type type);
struct ggml_tensor* ggml_new_tensor_1d(struct ggml_context*, enum ggml_type, int64_t);
struct ggml_tensor* ggml_new_tensor_2d(struct ggml_context*, enum ggml_type, int64_t, int64_t);
struct ggml_tensor* ggml_new_tensor_3d(struct ggml_context*, enum ggml_type, int64_t, int64_t, int64_t);
struct ggml_tensor* ggml_new_tensor_4d(struct ggml_context*, enum ggml_type, int64_t, int64_t, int64_t, int64_t);
struct ggml_tensor* ggml_dup_tensor(struct ggml_context*, const struct ggml_tensor*);
void ggml_set_input(struct ggml_tensor*);
struct ggml_tensor* ggml_view_3d(struct ggml_context*, struct ggml_tensor*, int64_t, int64_t, int64_t, size_t, size_t, size_t);
struct ggml_tensor* ggml_view_4d(struct ggml_context*, struct ggml_tensor*, int64_t, int64_t, int64_t, int64_t, size_t, size_t, size_t, size_t);
struct ggml_tensor* ggml_permute(struct ggml_context*, struct ggml_tensor*, int, int, int, int);
struct ggml_tensor* ggml_cont(struct ggml_context*, struct ggml_tensor*);
struct ggml_tensor* ggml_concat(struct ggml_context*, struct ggml_tensor*, struct ggml_tensor*, int);
struct ggml_tensor* ggml_neg(struct ggml_context*, struct ggml_tensor*);
struct ggml_tensor* ggml_add(struct ggml_context*, struct ggml_tensor*, struct ggml_tensor*);
struct ggml_tensor* ggml_mul(struct ggml_context*, struct ggml_tensor*, struct ggml_tensor*);
struct ggml_tensor* ggml_silu(struct ggml_context*, struct ggml_tensor*);
struct ggml_tensor* ggml_mul_mat(struct ggml_context*, struct ggml_tensor*, struct ggml_tensor*);
struct ggml_tensor* ggml_custom_4d(struct ggml_context*, enum ggml_type, int64_t, int64_t, int64_t, int64_t,
                                   struct ggml_tensor** args, int n_args, ggml_custom_op_t fun, int n_tasks, void* userdata);
#ifdef __cplusplus
}
#endif
