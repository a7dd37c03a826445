/*
 * nc.h — C ABI of the newch engine, implemented on NVIDIA B200 (sm_100a).
 *
 * This header declares the same entry points, enum values and struct layouts as newch's
 * engine/include/nc.h (v0.4.0), so the unchanged newch Python package (newch/_lib.py binds these
 * names by ctypes) and C programs written against newch link and run against the B200 library.
 * Each block cites the newch declaration it stands in for. The descriptions are of this
 * implementation: tensor data lives in B200 device memory, every op enqueues CUDA kernels on the
 * context's stream, and host pointers handed out by the data accessors are coherent mirrors.
 *
 * Memory: persistent tensors (parameters, optimizer state, BN buffers, anything created between
 * nc_persistent_begin/end) live until released or nc_free_ctx; temporaries live in a device step
 * arena that nc_step_end resets in O(1).
 * Errors: ops never abort; the first error sticks in the context and ops return NULL, and every
 * op passes NULL inputs through (newch nc.h:15-18). Errors found by a kernel (an out-of-range
 * label or index that could not be checked on the host) surface as NC_ERR_ARG at the next point
 * where the host waits for the device (nc_item, nc_copy_to, ...).
 */
#ifndef NC_H
#define NC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__) || defined(__clang__)
#define NC_API __attribute__((visibility("default")))
#else
#define NC_API
#endif

/* newch nc.h:40-42 */
#define NC_VERSION_MAJOR 0
#define NC_VERSION_MINOR 4
#define NC_VERSION_PATCH 0

/* newch nc.h:44-45 */
#define NC_MAX_DIMS 6
#define NC_ALL_AXES (-128)

/* newch nc.h:46-53 (values are part of the ABI) */
typedef enum { NC_F32 = 0, NC_I32 = 1, NC_F16 = 2, NC_I8 = 3, NC_U8 = 4, NC_DTYPE_COUNT } nc_dtype;

/* newch nc.h:55-58 */
typedef enum { NC_DEVICE_CPU = 0 } nc_device;

/* newch nc.h:60-67 */
typedef enum {
    NC_OK = 0,
    NC_ERR_SHAPE = 1,
    NC_ERR_DTYPE = 2,
    NC_ERR_OOM = 3,
    NC_ERR_ARG = 4,
    NC_ERR_STATE = 5
} nc_status;

typedef struct nc_ctx nc_ctx;
typedef struct nc_tensor nc_tensor;
typedef struct nc_module nc_module;
typedef struct nc_optim nc_optim;

/* ---- context: newch nc.h:78-107 ------------------------------------------------------------- */

/* Same layout as newch nc.h:78-83. arena_chunk_bytes is the minimum device-arena growth unit,
 * seed seeds the xoshiro256** stream (0 = the fixed default), force_reference = 1 selects the
 * strict FP32 (FFMA) GEMM path, threads is kept for host-side work only. */
typedef struct {
    size_t arena_chunk_bytes;
    uint64_t seed;
    int force_reference;
    int threads;
} nc_config;

NC_API nc_ctx *nc_init(const nc_config *cfg);      /* nc.h:85; binds the CUDA device (NC_DEVICE env, else 0) */
NC_API void nc_free_ctx(nc_ctx *ctx);              /* nc.h:86 */
NC_API void nc_manual_seed(nc_ctx *ctx, uint64_t seed); /* nc.h:87 */
NC_API void nc_step_end(nc_ctx *ctx);              /* nc.h:90: O(1) reset of the device step arena and tape */
NC_API void nc_arena_trim(nc_ctx *ctx);            /* nc.h:93: gives idle arena chunks back to the device pool */
NC_API int nc_num_threads(const nc_ctx *ctx);      /* nc.h:94 */
NC_API void nc_persistent_begin(nc_ctx *ctx);      /* nc.h:98 */
NC_API void nc_persistent_end(nc_ctx *ctx);        /* nc.h:99 */
NC_API int nc_set_grad_enabled(nc_ctx *ctx, int enabled); /* nc.h:102 */
NC_API int nc_ok(const nc_ctx *ctx);               /* nc.h:104 */
NC_API nc_status nc_status_code(const nc_ctx *ctx);/* nc.h:105 */
NC_API const char *nc_error(const nc_ctx *ctx);    /* nc.h:106 */
NC_API void nc_clear_error(nc_ctx *ctx);           /* nc.h:107 */

/* newch nc.h:109-114: byte counts of device memory */
typedef struct {
    size_t persistent_bytes;
    size_t arena_bytes_in_use;
    size_t arena_bytes_reserved;
    size_t arena_peak_bytes;
} nc_mem_stats;

NC_API nc_mem_stats nc_get_mem_stats(const nc_ctx *ctx); /* nc.h:116 */
NC_API void nc_reset_peak(nc_ctx *ctx);                  /* nc.h:117 */

/* ---- platform: newch nc.h:123-137 (host CPU facts; the kernel backend is "b200") ----------- */
typedef struct {
    const char *arch;
    int has_neon;
    int has_dotprod;
    int has_fp16;
    int has_avx2;
    int has_fma;
    int has_rvv;
    int n_cores;
    int n_big_cores;
} nc_cpu_info;

NC_API const nc_cpu_info *nc_cpu(const nc_ctx *ctx);    /* nc.h:135 */
NC_API const char *nc_kernel_backend(const nc_ctx *ctx); /* nc.h:136 */

/* ---- tensors: newch nc.h:143-190 ---------------------------------------------------------- */
NC_API nc_tensor *nc_empty(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_zeros(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_full(nc_ctx *ctx, float value, int ndim, const int64_t *shape);
/* Random tensors draw from the context's host-side xoshiro256** stream in element order, then
 * upload, so initial weights equal newch's bit for bit. */
NC_API nc_tensor *nc_randn(nc_ctx *ctx, float stddev, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_rand_uniform(nc_ctx *ctx, float lo, float hi, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_from_data(nc_ctx *ctx, nc_dtype dt, const void *data, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_scalar(nc_ctx *ctx, float value);
NC_API nc_tensor *nc_parameter(nc_ctx *ctx, const nc_tensor *init, int ndim, const int64_t *shape);

NC_API int nc_ndim(const nc_tensor *t);
NC_API int64_t nc_dim(const nc_tensor *t, int axis);
NC_API const int64_t *nc_shape(const nc_tensor *t);
NC_API int64_t nc_numel(const nc_tensor *t);
NC_API nc_dtype nc_get_dtype(const nc_tensor *t);
NC_API int nc_is_contiguous(const nc_tensor *t);
NC_API int nc_requires_grad(const nc_tensor *t);
NC_API int nc_is_persistent(const nc_tensor *t);
NC_API void nc_release(nc_tensor *t);
NC_API void nc_set_requires_grad(nc_tensor *t, int on);
NC_API nc_tensor *nc_grad(const nc_tensor *t);
NC_API void nc_set_name(nc_tensor *t, const char *name);
NC_API const char *nc_name(const nc_tensor *t);

/* newch nc.h:174-183. nc_data_f32/i32 return a host mirror of the tensor's device data (refreshed
 * by this call). Writes through it reach the device before the next op reads the tensor. A device
 * write after the call leaves an old pointer's contents stale: call again to refresh. */
NC_API float *nc_data_f32(nc_tensor *t);
NC_API int32_t *nc_data_i32(nc_tensor *t);
NC_API float nc_item(const nc_tensor *t);
NC_API float nc_get(const nc_tensor *t, const int64_t *index);
NC_API int nc_copy_to(const nc_tensor *t, void *dst, size_t dst_bytes);
NC_API int nc_copy_from(nc_tensor *t, const void *src, size_t src_bytes);
NC_API void nc_print(const nc_tensor *t);

/* ---- ops: newch nc.h:192-279 ---------------------------------------------------------------- */
NC_API nc_tensor *nc_add(nc_tensor *a, nc_tensor *b);
NC_API nc_tensor *nc_sub(nc_tensor *a, nc_tensor *b);
NC_API nc_tensor *nc_mul(nc_tensor *a, nc_tensor *b);
NC_API nc_tensor *nc_div(nc_tensor *a, nc_tensor *b);

NC_API nc_tensor *nc_neg(nc_tensor *x);
NC_API nc_tensor *nc_exp(nc_tensor *x);
NC_API nc_tensor *nc_log(nc_tensor *x);
NC_API nc_tensor *nc_sqrt(nc_tensor *x);
NC_API nc_tensor *nc_relu(nc_tensor *x);
NC_API nc_tensor *nc_sigmoid(nc_tensor *x);
NC_API nc_tensor *nc_tanh(nc_tensor *x);
NC_API nc_tensor *nc_scale(nc_tensor *x, float s);
NC_API nc_tensor *nc_add_scalar(nc_tensor *x, float s);
NC_API nc_tensor *nc_pow_scalar(nc_tensor *x, float p);

NC_API nc_tensor *nc_leaky_relu(nc_tensor *x, float negative_slope);
NC_API nc_tensor *nc_relu6(nc_tensor *x);
NC_API nc_tensor *nc_hardsigmoid(nc_tensor *x);
NC_API nc_tensor *nc_hardswish(nc_tensor *x);
NC_API nc_tensor *nc_silu(nc_tensor *x);
NC_API nc_tensor *nc_gelu(nc_tensor *x, int approximate_tanh);

NC_API nc_tensor *nc_matmul(nc_tensor *a, nc_tensor *b);
NC_API nc_tensor *nc_linear_fn(nc_tensor *x, nc_tensor *weight, nc_tensor *bias);

NC_API nc_tensor *nc_sum(nc_tensor *x, int axis, int keepdim);
NC_API nc_tensor *nc_mean(nc_tensor *x, int axis, int keepdim);
NC_API nc_tensor *nc_max(nc_tensor *x, int axis, int keepdim);

NC_API nc_tensor *nc_reshape(nc_tensor *x, int ndim, const int64_t *shape);
NC_API nc_tensor *nc_transpose(nc_tensor *x, int axis0, int axis1);
NC_API nc_tensor *nc_slice(nc_tensor *x, int axis, int64_t start, int64_t length, int64_t step);
NC_API nc_tensor *nc_contiguous(nc_tensor *x);
NC_API nc_tensor *nc_index_select(nc_tensor *x, nc_tensor *idx);

NC_API nc_tensor *nc_conv2d(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, int stride_h, int stride_w,
                            int pad_h, int pad_w);
NC_API nc_tensor *nc_conv2d_ex(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, int stride_h, int stride_w,
                               int pad_h, int pad_w, int dilation_h, int dilation_w, int groups);
NC_API nc_tensor *nc_max_pool2d(nc_tensor *x, int k_h, int k_w, int stride_h, int stride_w, int pad_h, int pad_w);
NC_API nc_tensor *nc_avg_pool2d(nc_tensor *x, int k_h, int k_w, int stride_h, int stride_w, int pad_h, int pad_w);

/* Draws one value per element from the context's xoshiro256** stream, in element order, on the
 * device (jump-ahead), so masks equal newch's for the same seed and call order. */
NC_API nc_tensor *nc_dropout(nc_tensor *x, float p);

NC_API nc_tensor *nc_batch_norm(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, nc_tensor *running_mean,
                                nc_tensor *running_var, int training, float momentum, float eps);

NC_API nc_tensor *nc_log_softmax(nc_tensor *x);
NC_API nc_tensor *nc_softmax(nc_tensor *x);
NC_API nc_tensor *nc_layer_norm(nc_tensor *x, int normalized_ndim, nc_tensor *weight, nc_tensor *bias, float eps);
NC_API nc_tensor *nc_masked_fill(nc_tensor *x, nc_tensor *mask, float value);
NC_API nc_tensor *nc_cross_entropy(nc_tensor *logits, nc_tensor *labels);
NC_API nc_tensor *nc_mse_loss(nc_tensor *pred, nc_tensor *target);
NC_API nc_tensor *nc_nll_loss(nc_tensor *logp, nc_tensor *labels, int sum);

NC_API nc_tensor *nc_argmax(nc_tensor *x, int axis);
NC_API nc_tensor *nc_detach(nc_tensor *x);

/* newch nc.h:279 */
typedef enum { NC_CMP_EQ, NC_CMP_NE, NC_CMP_LT, NC_CMP_LE, NC_CMP_GT, NC_CMP_GE } nc_cmp;
NC_API nc_tensor *nc_compare(nc_tensor *a, nc_tensor *b, nc_cmp op);
NC_API nc_tensor *nc_cat(int n, nc_tensor *const *xs, int axis);
NC_API nc_tensor *nc_to_dtype(nc_tensor *x, nc_dtype dt);

/* ---- int8 quantization: newch nc.h:292-298 ------------------------------------------------- */
NC_API nc_tensor *nc_quantize_rows(nc_tensor *w, nc_tensor **scale);
NC_API nc_tensor *nc_linear_int8(nc_tensor *x, nc_tensor *wq, nc_tensor *w_scale, nc_tensor *bias);

/* ---- serialization: newch nc.h:304-307 (NCW1 files, docs/FORMAT.md of newch) ------------------ */
NC_API nc_status nc_save(nc_ctx *ctx, const char *path, int n, const char *const *names, nc_tensor *const *tensors);
NC_API nc_status nc_load(nc_ctx *ctx, const char *path, int n, const char *const *names, nc_tensor *const *tensors);

/* ---- autograd: newch nc.h:313-346 ------------------------------------------------------------- */
NC_API nc_status nc_backward(nc_tensor *loss);
enum { NC_BACKWARD_FREE_GRAPH = 1, NC_BACKWARD_RETAIN = 2 };
NC_API void nc_release_temp(nc_tensor *t);
NC_API nc_status nc_backward_ex(nc_tensor *loss, int flags, nc_tensor *const *keep, int n_keep);
NC_API void nc_zero_grad(nc_tensor *t);
NC_API void nc_clear_grad(nc_tensor *t);

typedef nc_tensor *(*nc_scalar_fn)(nc_ctx *ctx, nc_tensor **inputs, void *user);
NC_API float nc_gradcheck(nc_ctx *ctx, nc_scalar_fn fn, nc_tensor **inputs, int n_inputs, void *user, float eps);

/* ---- C-side modules: newch nc.h:352-366 ------------------------------------------------------ */
typedef enum { NC_ACT_RELU, NC_ACT_SIGMOID, NC_ACT_TANH } nc_activation;
NC_API nc_module *nc_linear(nc_ctx *ctx, int64_t in_features, int64_t out_features, int bias);
NC_API nc_module *nc_act(nc_ctx *ctx, nc_activation kind);
NC_API nc_module *nc_sequential(nc_ctx *ctx, int n, nc_module **mods);
NC_API nc_tensor *nc_forward(nc_module *m, nc_tensor *x);
NC_API int nc_parameters(nc_module *m, nc_tensor **out, int max);
NC_API const char *nc_module_name(const nc_module *m);
NC_API void nc_set_training(nc_module *m, int training);

/* ---- optimizers: newch nc.h:370-411 ---------------------------------------------------------- */
/* Same layout as newch nc.h:370-375. */
typedef struct {
    float lr;
    float momentum;
    float weight_decay;
    float beta1, beta2, eps;
} nc_optim_opts;

/* One fused kernel updates every parameter. With NC_WORLD_SIZE > 1 (see nc_ext.h) the gradients
 * are summed across ranks by one NCCL all-reduce of the flat gradient buffer before the update. */
NC_API nc_optim *nc_sgd(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts);
NC_API nc_optim *nc_adam(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts);
NC_API nc_optim *nc_adamw(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts);
NC_API nc_optim *nc_rmsprop(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts, int eps_inside_sqrt);
NC_API void nc_optim_zero_grad(nc_optim *o);
NC_API void nc_optim_clear_grad(nc_optim *o);
NC_API void nc_optim_step(nc_optim *o);
NC_API void nc_optim_free(nc_optim *o);
NC_API void nc_optim_set_lr(nc_optim *o, float lr);
/* Host mirror of the state slot (refreshed by this call; writes reach the device before the next
 * nc_optim_step). */
NC_API float *nc_optim_state(nc_optim *o, int param, int slot);
NC_API int64_t nc_optim_get_step(const nc_optim *o);
NC_API void nc_optim_set_step(nc_optim *o, int64_t t);
NC_API void nc_optim_set_opts(nc_optim *o, nc_optim_opts opts);
NC_API void nc_optim_set_accumulation(nc_optim *o, int steps);
NC_API float nc_clip_grad_norm(nc_tensor **params, int n, float max_norm);

#ifdef __cplusplus
}
#endif

#endif /* NC_H */
