/* Internal definitions of the B200 engine (host C11). Not installed.
 *
 * The engine keeps newch's execution model (engine/src/core/nc_internal.h:34-105 of newch): eager
 * ops through one entry point, a tape of nodes walked newest-first for backward, a step arena reset
 * in O(1). What differs is where things live:
 *   - tensor data is device memory (B200 HBM): a device step arena for temporaries, the CUDA
 *     stream-ordered pool for persistent tensors;
 *   - tensor headers, tape nodes and op-private records are host memory in a host step arena;
 *   - host views of device data are explicit mirrors with a coherence state per data owner.
 */
#ifndef NC_INTERNAL_H
#define NC_INTERNAL_H

#include "../../include/nc.h"
#include "../../include/nc_ext.h"
#include "nck.h"

#include <stdarg.h>
#include <string.h>

#define NC_DEV_ALIGN 256        /* device allocations: TMA / vector loads / coalescing friendly */
#define NC_HOST_ALIGN 64
#define NC_MAX_INPUTS 6
#define NC_MIN_DEV_CHUNK ((size_t)64 << 20)
#define NC_HOST_CHUNK ((size_t)1 << 20)
#define NC_MIRROR_SMALL 4096    /* owners up to this many bytes keep an eager host mirror */

/* ---- tensor ----------------------------------------------------------------------------------- */

enum {
    NC_TF_REQUIRES_GRAD = 1u << 0,
    NC_TF_PERSISTENT = 1u << 1,
    NC_TF_OWNS_DATA = 1u << 2,
    NC_TF_GRAD_CLEARED = 1u << 3,
    NC_TF_ON_TAPE = 1u << 4,
};

/* coherence of an owner's host mirror */
enum {
    NC_COH_HOST_VALID = 1u << 0, /* mirror equals device data */
    NC_COH_HOST_DIRTY = 1u << 1, /* mirror handed out: may hold writes the device has not seen */
};

typedef struct nc_node nc_node;

struct nc_tensor {
    nc_ctx *ctx;
    nc_dtype dtype;
    int ndim;
    uint32_t flags;
    int64_t shape[NC_MAX_DIMS];
    int64_t stride[NC_MAX_DIMS];
    void *data;        /* device address of logical element 0 */
    nc_tensor *grad;   /* contiguous f32, same logical shape */
    nc_node *node;
    nc_tensor *owner;  /* views: the tensor whose data this aliases */
    const char *name;
    /* owners only */
    size_t bytes;      /* size of the data allocation */
    void *host;        /* host mirror of the whole allocation (NULL until needed) */
    uint32_t coh;
    int host_pinned;   /* mirror came from cudaMallocHost */
    /* leaves during a backward pass: writers of this tensor's gradient still to run */
    uint32_t bw_epoch;
    int32_t bw_pending;
    /* parameters registered with an optimizer: the optimizer and the parameter's index in it */
    struct nc_optim *optim;
    int32_t optim_slot;
    /* owners whose values are still a pending epilogue (not written yet; fusion.c) */
    struct nc_deferred *deferred;
    /* live consumers of this tensor in the current backward pass */
    uint32_t use_epoch;
    int32_t uses;
};

/* ---- op registry ------------------------------------------------------------------------------ */

/* NC_OPF_RECIPE: the op's forward takes a pending recipe as input itself (fusion.c) instead of having
 * nc__apply materialise it first */
enum {
    NC_OPF_ELEMENTWISE = 1u << 0,
    NC_OPF_REDUCTION = 1u << 1,
    NC_OPF_VIEW = 1u << 2,
    NC_OPF_NONDIFF = 1u << 3,
    NC_OPF_RECIPE = 1u << 4
};

typedef struct {
    int64_t i[NC_MAX_DIMS + 2];
    float f[4];
} nc_op_params;

typedef struct nc_op_def {
    const char *name;
    uint32_t flags;
    int kind;
    nc_status (*infer)(nc_node *n, nc_dtype *dt, int *ndim, int64_t *shape);
    int (*view)(nc_node *n, int ndim, const int64_t *shape);
    nc_status (*forward)(nc_node *n);
    void (*backward)(nc_node *n);
} nc_op_def;

struct nc_node {
    const nc_op_def *op;
    nc_tensor *in[NC_MAX_INPUTS];
    int n_in;
    nc_tensor *out;
    nc_op_params p;
    void *saved;       /* op-private host record (host arena); may point at device scratch */
    nc_node *prev;     /* the step's record log, newest first */
    uint64_t seq;      /* recording order within the context */
    uint32_t mark;     /* backward epoch in which the node was found live */
    uint32_t fused;    /* backward epoch in which a fused chain already ran this node's backward */
    int released;
};

#define NC_OP_LIST(X)                                                          \
    X(add) X(sub) X(mul) X(div)                                                \
    X(neg) X(exp) X(log) X(sqrt) X(relu) X(sigmoid) X(tanh)                    \
    X(scale) X(add_scalar) X(pow_scalar)                                       \
    X(leaky_relu) X(relu6) X(hardsigmoid) X(hardswish) X(silu) X(gelu)         \
    X(gelu_tanh)                                                               \
    X(matmul) X(linear)                                                        \
    X(sum) X(mean) X(max) X(argmax)                                            \
    X(reshape) X(transpose) X(contiguous) X(detach) X(index_select)            \
    X(log_softmax) X(softmax) X(cross_entropy)                                 \
    X(conv2d) X(max_pool2d) X(avg_pool2d) X(dropout) X(batch_norm)             \
    X(linear_int8) X(nll_loss) X(compare) X(cat) X(to_dtype)                   \
    X(bmm) X(layer_norm) X(masked_fill) X(slice)

#define NC_DECLARE_OP(name) extern const nc_op_def nc_op_##name;
NC_OP_LIST(NC_DECLARE_OP)
#undef NC_DECLARE_OP

int nc__op_count(void);
const nc_op_def *nc__op_at(int i);

nc_tensor *nc__apply(const nc_op_def *op, nc_tensor **in, int n_in, const nc_op_params *p);

/* ---- context ---------------------------------------------------------------------------------- */

typedef struct nc_hchunk {
    struct nc_hchunk *next;
    size_t cap, used;
    unsigned char *base;
} nc_hchunk;

typedef struct {
    char *base;
    size_t cap, used;
} nc_dchunk;

typedef struct {
    char *p;
    size_t size;
} nc_dfree;


struct nc_ctx {
    /* device */
    nck_dev dev;
    char device_name[128];
    int device_ok;

    /* device step arena: bump chunks + best-fit free list of released blocks */
    nc_dchunk *dchunks;
    int n_dchunks, cap_dchunks;
    int cur_dchunk;
    nc_dfree *dfree;
    int n_dfree, cap_dfree;
    size_t dchunk_min;
    size_t arena_in_use, arena_reserved, arena_peak;

    /* host step arena for headers, nodes and op records */
    nc_hchunk *hchunks, *hcur;

    /* persistent device blocks (open-addressing set of device pointers) */
    size_t persistent_bytes;
    void **pmem;
    size_t pmem_cap, pmem_n;

    /* backward temporaries of the node being processed */
    void *bwd_tmp[64];
    size_t bwd_tmp_size[64];
    int bwd_tmp_n;
    int bwd_logging;
    int grad_alloc;
    uint32_t mark_epoch;
    uint64_t node_seq;

    int persistent_depth;
    int grad_enabled;
    nc_node *tape;
    int fwd_on_tape;   /* the op whose forward is running will be recorded */
    int fuse;          /* deferred epilogues and fused backward chains (NC_FUSE=0: off) */
    struct nc_deferred *deferred_head;

    nc_status status;
    char err[256];

    uint64_t rng[4];
    uint64_t rng_count;       /* draws taken from the stream since it was seeded */
    uint64_t rng_step_start;  /* rng_count at the start of the current step */
    int64_t dp_rng_stride;    /* data parallel: draws of one micro-batch step (0: streams not interleaved) */
    nc_cpu_info cpu;
    int n_threads;
    int force_reference;

    /* pinned staging ring for small uploads */
    unsigned char *stage;
    size_t stage_cap, stage_pos;
    void *stage_events[32];
    int stage_slot;

    /* data parallel */
    int dp_rank, dp_world;
    void *nccl_comm;
    void *comm_stream;   /* cudaStream_t of the gradient all-reduces (created with the communicator) */
    void *ev_main;       /* cudaEvent_t: main-stream point a reduce waits for */
    void *ev_comm;       /* cudaEvent_t: comm-stream point the main stream waits for */
    int comm_pending;    /* reduces enqueued on comm_stream since the last join */
    /* dropout keep masks drawn on a side stream (rng.c): they depend on no tensor, so they run while
     * the main stream is still busy with earlier work; the main stream waits before each consumer */
    void *side_stream;   /* cudaStream_t, created on first use; NULL: masks drawn on the main stream */
    void *ev_side;       /* cudaEvent_t: a mask is drawn */
    void *ev_step;       /* cudaEvent_t: recorded at nc_step_end, waited for by the next step's masks */
    unsigned char *side_pool; /* device block for the step's masks and tables (bump, reset at step end) */
    size_t side_cap, side_used;
    int side_fresh;      /* no mask drawn yet this step: wait for ev_step first */
    int side_off;        /* NC_RNG_SIDE=0, or set-up failed */
    int side_all;        /* NC_RNG_SIDE=1: every mask on the side stream, whatever its size */
    struct nc_optim *optims; /* optimizers of this context (intrusive list) */
    /* data parallel BatchNorm: each training forward stages its batch (mean, unbiased variance) here;
     * nc__dp_bn_flush gathers every rank's and applies the running-statistic updates in rank order */
    float *bn_stage, *bn_gather;
    int64_t bn_stage_cap, bn_stage_used;
    struct nc_bn_pending *bn_pending;
    int bn_n, bn_cap;
    void *bn_table_dev;
    int bn_table_cap;

    /* scratch double accumulators etc. */
    double *dscratch;
};

void *nc__arena_alloc(nc_ctx *ctx, size_t bytes);             /* device, step lifetime */
void nc__arena_free(nc_ctx *ctx, void *p, size_t bytes);
void *nc__persistent_alloc(nc_ctx *ctx, size_t bytes);        /* device */
void nc__persistent_free(nc_ctx *ctx, void *p, size_t bytes);
void *nc__alloc(nc_ctx *ctx, size_t bytes, int persistent);
void *nc__meta_alloc(nc_ctx *ctx, size_t bytes, int persistent); /* host headers/records */
void nc__meta_free(nc_ctx *ctx, void *p, int persistent);
int nc__is_persistent_mode(const nc_ctx *ctx);

void nc__error(nc_ctx *ctx, nc_status code, const char *fmt, ...);
/* checks the last CUDA call; on failure records NC_ERR_STATE and returns 0 */
int nc__cuda_ok(nc_ctx *ctx, int cuda_err, const char *what);
/* waits for the stream, folds kernel-found errors into the context status; returns 1 if ok */
int nc__sync(nc_ctx *ctx);

uint64_t nc__rng_next(nc_ctx *ctx);
float nc__rand_uniform01(nc_ctx *ctx);
float nc__rand_normal(nc_ctx *ctx);
/* advances the context stream by n draws without producing them */
void nc__rng_skip(nc_ctx *ctx, uint64_t n);
int nc__rng_device_init(nc_ctx *ctx);
const uint64_t *nc__rng_run_polys(int64_t count);          /* x^(64 k) mod P, k < count (host) */
const void *nc__rng_dropout_table(nc_ctx *ctx, int64_t n); /* the same on the device, or NULL */
/* the dropout kernel's Horner window tables for the current state, on the device (32 KiB), or NULL */
const void *nc__rng_dropout_tabs(nc_ctx *ctx);
/* the window tables for state s0 on the host: 1024 entries of four words */
void nc__rng_build_tabs(const uint64_t s0[4], uint64_t (*tab)[4]);

void nc__detect_cpu(nc_cpu_info *info);

/* host <-> device */
void nc__upload(nc_ctx *ctx, void *dst, const void *src, size_t bytes);
/* the same on another stream of the context (void * = cudaStream_t) */
void nc__upload_on(nc_ctx *ctx, void *stream, void *dst, const void *src, size_t bytes);
/* Draws the keep mask of the stream's next n draws (threshold p) on the side stream into a block of
 * the step's side pool and makes the main stream wait for it; *bits receives the block. Returns 0
 * (nothing drawn) when the side stream is off, per-kernel timing is on or the pool is full: the
 * caller draws on the main stream. The caller advances the stream past the n draws either way. */
int nc__rng_side_mask(nc_ctx *ctx, int64_t n, float p, uint32_t **bits);
void nc__rng_side_step_end(nc_ctx *ctx);
void nc__rng_side_free(nc_ctx *ctx);
void nc__download(nc_ctx *ctx, void *dst, const void *src, size_t bytes); /* synchronous */

/* ---- tensor helpers --------------------------------------------------------------------------- */

size_t nc__dtype_size(nc_dtype dt);
const char *nc__dtype_name(nc_dtype dt);
int64_t nc__shape_numel(int ndim, const int64_t *shape);
void nc__contig_strides(int ndim, const int64_t *shape, int64_t *stride);
int nc__norm_axis(int axis, int ndim);
int nc__same_shape(const nc_tensor *a, const nc_tensor *b);
const char *nc__shape_str(int ndim, const int64_t *shape, char *buf, size_t size);
int nc__expect_f32(const nc_node *n, int i);

nc_tensor *nc__tensor_new(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape, int persistent);
nc_tensor *nc__tensor_alias(const nc_tensor *src, int persistent);
static inline nc_tensor *nc__owner(nc_tensor *t) { return t->owner ? t->owner : t; }

nc_tensor *nc__grad_buf(nc_tensor *t);
/* The gradient buffer for a writer that sets every element of it: a new (or zero_grad-cleared)
 * buffer of a temporary comes back without zero-filling and *acc = 0 (the writer stores); otherwise
 * *acc = 1 (the writer adds). Persistent tensors always get a zero-filled buffer and *acc = 1. */
nc_tensor *nc__grad_buf_acc(nc_tensor *t, int *acc);
static inline int nc__needs_grad(const nc_tensor *t) { return (t->flags & NC_TF_REQUIRES_GRAD) != 0; }
/* A backward whose input gradient is its output gradient element for element in row-major order (a
 * reshape, a contiguous copy) passes the buffer on instead of copying it, when the input has no
 * gradient yet and is a temporary and the pass frees gradients as it goes. Returns 1 when done. */
int nc__grad_handoff(nc_tensor *in, nc_tensor *out);

/* device pointer to t's element 0 after pushing any host writes to the device */
void *nc__dev(nc_tensor *t);
/* t (its owner) is about to be written by a kernel: host mirror no longer valid */
void nc__dev_write(nc_tensor *t);
/* contiguous device f32 data of t (a copy in the arena when t is a strided view) */
const float *nc__contig_f32(nc_tensor *t);
/* contiguous device data of any dtype */
const void *nc__contig(nc_tensor *t);
/* host copy of t's contiguous data (mirror when valid, else a download); NULL on error */
const void *nc__host_view(nc_tensor *t);

void nc__bcast_strides(const nc_tensor *t, int ndim, const int64_t *shape, int64_t *out);
void nc__bcast_strides_shape(int tn, const int64_t *tshape, int ndim, const int64_t *shape, int64_t *out);

static inline nck_dev *nc__k(nc_ctx *ctx) { return &ctx->dev; }

/* GEMM entry point for ops (same contract as the newch kernel table's gemm_f32, newch
 * engine/src/kernels/kernels.h:34-41, plus batch strides) */
void nc__gemm(nc_ctx *ctx, int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
              int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc);
void nc__gemm_batched(nc_ctx *ctx, const nck_gemm_args *a);

/* data parallel: all-reduce of a device float buffer, averaged over ranks (on the main stream) */
int nc__dp_allreduce_mean(nc_ctx *ctx, float *buf, int64_t n);
/* dst = mean over ranks of src, enqueued on the communication stream after the main stream's work so
 * far; nc__dp_join makes the main stream wait for every such reduce */
int nc__dp_reduce_async(nc_ctx *ctx, const float *src, float *dst, int64_t n);
/* elementwise maximum over ranks of a byte buffer, in place, on the communication stream */
int nc__dp_max_bytes_async(nc_ctx *ctx, unsigned char *buf, int64_t n);
void nc__dp_join(nc_ctx *ctx);
/* data-parallel BatchNorm running statistics (dp.c): staging of one training forward's statistics
 * (returns the device address for 2 * C floats: means, then unbiased variances), and the flush */
float *nc__dp_bn_stage(nc_ctx *ctx, float *running_mean, float *running_var, int64_t C, float momentum);
int nc__dp_bn_flush(nc_ctx *ctx, int on_comm_stream);
/* data-parallel dropout streams at a step boundary (dp.c) */
void nc__dp_rng_step_end(nc_ctx *ctx);

/* ---- deferred epilogues (fusion.c) -------------------------------------------------------------
 * A BatchNorm output in training, and an activation of it, can be left unwritten: the tensor holds a
 * recipe (act(BatchNorm(x)) with the batch statistics) until something reads it. A 2 x 2 max pool
 * reads the recipe and pools straight from x; anything else that touches the data materialises it
 * first (nc__dev and the host paths call nc__materialize). In backward, a pool or activation over
 * such a chain runs the whole chain's backward in one fused BatchNorm backward. */
enum { NC_DEF_BN = 0, NC_DEF_ATTN = 1, NC_DEF_UNARY = 2 };
typedef struct nc_deferred {
    nc_tensor *owner;              /* the tensor whose values are pending */
    nc_tensor *src[3];             /* owners whose data feeds the recipe (NULL: unused) */
    int kind;                      /* NC_DEF_* */
    /* NC_DEF_BN: act(BatchNorm(x)) */
    const float *x, *w, *b, *mean, *invstd;
    int64_t N, C, S;
    int act;                       /* NCK_UN_* kind applied after the normalisation, -1: none */
    float act_s;
    /* NC_DEF_ATTN: a tensor of the scores -> mask -> softmax -> dropout chain (at.stage says which) */
    nck_attn at;
    /* NC_DEF_UNARY: act(x) over N = numel contiguous elements (x, act, act_s above); adopt: the
     * source's arena block when the caller released the source first (freed with the recipe) */
    void *adopt;
    size_t adopt_bytes;
    struct nc_deferred *next;
} nc_deferred;

void nc__defer_bn(nc_ctx *ctx, nc_tensor *out, nc_tensor *x, const float *X, const float *w, const float *b,
                  const float *mean, const float *invstd, int64_t N, int64_t C, int64_t S);
/* the pending recipe of t when t is the whole (owner) tensor, else NULL */
const nc_deferred *nc__deferred_of(const nc_tensor *t);
/* out (a fresh tensor of t's shape) := act(t) as a recipe when t is pending and act fuses */
int nc__defer_act(nc_tensor *out, nc_tensor *t, int act, float act_s);
void nc__materialize(nc_tensor *owner);
/* owner's data is about to be freed or overwritten: recipes reading it are materialised first, its
 * own recipe (if any) is dropped */
void nc__deferred_release(nc_tensor *owner);
void nc__deferred_flush(nc_ctx *ctx);  /* materialise every pending recipe */
void nc__deferred_reset(nc_ctx *ctx);  /* step end: forget every recipe (their storage is reset) */
/* Attention chains (fusion.c). Each returns 1 when it took the op (out is a recipe, or was computed
 * by the fused kernel), 0 when the op runs its own kernels. */
/* out := act(x) as a recipe (no tape: an inference forward), for a consumer that applies act itself
 * (the int8 linear's quantization); 1 when deferred */
int nc__defer_unary(nc_tensor *out, nc_tensor *x, int act, float act_s);
/* owner (a temporary being released) feeds only a pending unary recipe: the recipe takes over its
 * data block (freed when the recipe is computed or dropped); 1 when it did */
int nc__deferred_adopt(nc_tensor *owner);
/* t's pending unary recipe (its input data, kind, parameter), or 0 */
int nc__unary_recipe(const nc_tensor *t, const float **x, int *act, float *act_s);
int nc__attn_bmm(nc_node *n);                       /* scores q @ k^T, or probabilities @ v */
int nc__attn_mask(nc_node *n);                      /* masked_fill of the scores */
int nc__attn_softmax(nc_node *n);                   /* softmax of the (masked) scores */
int nc__attn_scale(nc_node *n, float s);            /* scale of the scores */
/* dropout of the probabilities: bits holds the keep mask (the caller drew it from the stream) */
int nc__attn_dropout_ok(const nc_tensor *x); /* x is probabilities a dropout can extend */
int nc__attn_dropout(nc_node *n, const uint32_t *bits);
/* Runs the fused backward of the chain that ends at node n when there is one: fills consumed (room
 * for NC_CHAIN_MAX) with the chain's other nodes (whose own backward must not run) and returns their
 * count, else 0. */
#define NC_CHAIN_MAX 6
/* x at each window's argmax when a max pool ran over a BatchNorm recipe (ops_conv.c), else NULL */
const float *nc__pool_xarg(const nc_node *n);
int nc__fused_backward(nc_ctx *ctx, nc_node *n, nc_node **consumed);
/* the values of n's output and inputs, for a backward that reads them: pending recipes computed */
void nc__backward_inputs(nc_node *n);
/* the NCK_UN_* kind of a unary activation op, -1 for any other op (ops_elementwise.c) */
int nc__unary_kind(const nc_op_def *op);

/* Backward-pass gradient readiness of optimizer parameters (optim.c). A backward pass announces each
 * leaf whose gradient it will write (nc__grad_expect, once per leaf per pass) and reports it final
 * after its last writer has been enqueued (nc__grad_final); nc__grad_pass_begin opens a pass. They
 * let data-parallel runs all-reduce gradient buckets while the rest of the pass is still running. */
void nc__grad_pass_begin(nc_ctx *ctx);
void nc__grad_expect(nc_tensor *leaf);
void nc__grad_final(nc_tensor *leaf);

#endif /* NC_INTERNAL_H */
