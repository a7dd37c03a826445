/* Tensors: creation, accessors, host mirrors, strided copies, gradient buffers, op registry.
 *
 * Semantics follow newch engine/src/core/tensor.c (creation :120-207, accessors :209-307,
 * grad buffers :375-388). Data lives on the device; host access goes through a per-owner mirror:
 *   HOST_VALID  the mirror equals the device data (reads need no device round trip);
 *   HOST_DIRTY  the mirror was handed out by nc_data_f32/i32 and may hold host writes: the next
 *               device use of the tensor uploads it first (nc__dev).
 * Small owners (<= NC_MIRROR_SMALL bytes) keep a mirror from birth so scalars such as BatchNorm's
 * num_batches_tracked are read and written by the host without waiting for the device.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

/* ---- shape helpers ---------------------------------------------------------------------------- */

size_t nc__dtype_size(nc_dtype dt) {
    switch (dt) {
    case NC_F32:
    case NC_I32: return 4;
    case NC_F16: return 2;
    case NC_I8:
    case NC_U8: return 1;
    default: return 0;
    }
}

const char *nc__dtype_name(nc_dtype dt) {
    static const char *names[] = {"f32", "i32", "f16", "i8", "u8"};
    return (dt >= 0 && dt < NC_DTYPE_COUNT) ? names[dt] : "?";
}

int64_t nc__shape_numel(int ndim, const int64_t *shape) {
    int64_t n = 1;
    for (int i = 0; i < ndim; i++) n *= shape[i];
    return n;
}

void nc__contig_strides(int ndim, const int64_t *shape, int64_t *stride) {
    int64_t s = 1;
    for (int i = ndim - 1; i >= 0; i--) {
        stride[i] = s;
        s *= shape[i];
    }
}

int nc__norm_axis(int axis, int ndim) {
    if (axis < 0) axis += ndim;
    return (axis >= 0 && axis < ndim) ? axis : -1;
}

int nc__same_shape(const nc_tensor *a, const nc_tensor *b) {
    if (a->ndim != b->ndim) return 0;
    for (int i = 0; i < a->ndim; i++)
        if (a->shape[i] != b->shape[i]) return 0;
    return 1;
}

const char *nc__shape_str(int ndim, const int64_t *shape, char *buf, size_t size) {
    size_t pos = (size_t)snprintf(buf, size, "[");
    for (int i = 0; i < ndim && pos < size; i++)
        pos += (size_t)snprintf(buf + pos, size - pos, i ? ", %lld" : "%lld", (long long)shape[i]);
    if (pos < size) snprintf(buf + pos, size - pos, "]");
    return buf;
}

int nc__expect_f32(const nc_node *n, int i) {
    if (n->in[i]->dtype == NC_F32) return 1;
    nc__error(n->in[i]->ctx, NC_ERR_DTYPE, "%s: input %d must be f32, got %s", n->op->name, i,
              nc__dtype_name(n->in[i]->dtype));
    return 0;
}

void nc__bcast_strides_shape(int tn, const int64_t *tshape, int ndim, const int64_t *shape, int64_t *out) {
    int64_t ts[NC_MAX_DIMS];
    nc__contig_strides(tn, tshape, ts);
    for (int i = 0; i < ndim; i++) {
        int j = i - (ndim - tn);
        out[i] = (j < 0 || (tshape[j] == 1 && shape[i] != 1)) ? 0 : ts[j];
    }
}

void nc__bcast_strides(const nc_tensor *t, int ndim, const int64_t *shape, int64_t *out) {
    for (int i = 0; i < ndim; i++) {
        int j = i - (ndim - t->ndim);
        out[i] = (j < 0 || (t->shape[j] == 1 && shape[i] != 1)) ? 0 : t->stride[j];
    }
}

/* ---- mirrors ---------------------------------------------------------------------------------- */


/* host mirror buffer of an owner, allocated on first use */
static void *mirror_of(nc_tensor *o) {
    if (o->host) return o->host;
    size_t bytes = o->bytes ? o->bytes : 1;
    if (o->flags & NC_TF_PERSISTENT) {
        void *p = NULL;
        if (bytes >= ((size_t)1 << 16) && cudaMallocHost(&p, bytes) == cudaSuccess) {
            o->host_pinned = 1;
        } else {
            cudaGetLastError();
            p = malloc(bytes);
            o->host_pinned = 0;
        }
        o->host = p;
    } else {
        o->host = nc__meta_alloc(o->ctx, bytes, 0);
        o->host_pinned = 0;
    }
    if (!o->host) nc__error(o->ctx, NC_ERR_OOM, "out of host memory (mirror, %zu bytes)", bytes);
    return o->host;
}

static void mirror_free(nc_tensor *o) {
    if (!o->host || !(o->flags & NC_TF_PERSISTENT)) return;
    if (o->host_pinned) cudaFreeHost(o->host);
    else free(o->host);
    o->host = NULL;
}

/* makes the owner's mirror hold the device data; returns it */
static void *mirror_refresh(nc_tensor *o) {
    if (o->deferred) nc__materialize(o);
    void *h = mirror_of(o);
    if (!h) return NULL;
    if (!(o->coh & NC_COH_HOST_VALID)) {
        nc__download(o->ctx, h, o->data, o->bytes);
        if (o->ctx->status != NC_OK) return NULL;
        o->coh |= NC_COH_HOST_VALID;
    }
    return h;
}

void *nc__dev(nc_tensor *t) {
    nc_tensor *o = nc__owner(t);
    if (o->deferred) nc__materialize(o);
    if (o->coh & NC_COH_HOST_DIRTY) {
        nc__upload(o->ctx, o->data, o->host, o->bytes);
        o->coh &= ~NC_COH_HOST_DIRTY;
    }
    return t->data;
}

void nc__dev_write(nc_tensor *t) {
    nc_tensor *o = nc__owner(t);
    if (o->deferred) nc__materialize(o);
    if (o->coh & NC_COH_HOST_DIRTY) nc__dev(o);
    o->coh &= ~NC_COH_HOST_VALID;
}

const void *nc__host_view(nc_tensor *t) {
    nc_tensor *o = nc__owner(t);
    if (o->deferred || !(o->coh & NC_COH_HOST_VALID) || !o->host || !nc_is_contiguous(t)) return NULL;
    return (const char *)o->host + ((const char *)t->data - (const char *)o->data);
}

/* ---- creation --------------------------------------------------------------------------------- */

static int check_shape(nc_ctx *ctx, int ndim, const int64_t *shape) {
    if (ndim < 0 || ndim > NC_MAX_DIMS) {
        nc__error(ctx, NC_ERR_SHAPE, "ndim %d out of range [0, %d]", ndim, NC_MAX_DIMS);
        return 0;
    }
    const int64_t limit = INT64_MAX / 8;
    int64_t n = 1;
    for (int i = 0; i < ndim; i++) {
        if (shape[i] < 0) {
            nc__error(ctx, NC_ERR_SHAPE, "negative dimension %lld", (long long)shape[i]);
            return 0;
        }
        if (shape[i] && n > limit / shape[i]) {
            char sb[160];
            nc__error(ctx, NC_ERR_SHAPE, "shape %s has too many elements", nc__shape_str(ndim, shape, sb, sizeof sb));
            return 0;
        }
        n *= shape[i];
    }
    return 1;
}

nc_tensor *nc__tensor_new(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape, int persistent) {
    if (!ctx || !check_shape(ctx, ndim, shape)) return NULL;
    if (nc__dtype_size(dt) == 0) {
        nc__error(ctx, NC_ERR_DTYPE, "unknown dtype %d", (int)dt);
        return NULL;
    }
    nc_tensor *t = (nc_tensor *)nc__meta_alloc(ctx, sizeof(nc_tensor), persistent);
    if (!t) return NULL;
    t->ctx = ctx;
    t->dtype = dt;
    t->ndim = ndim;
    if (ndim) memcpy(t->shape, shape, (size_t)ndim * sizeof(int64_t));
    nc__contig_strides(ndim, t->shape, t->stride);
    t->bytes = (size_t)nc__shape_numel(ndim, shape) * nc__dtype_size(dt);
    t->data = nc__alloc(ctx, t->bytes, persistent);
    if (!t->data) {
        if (persistent) free(t);
        return NULL;
    }
    t->flags |= NC_TF_OWNS_DATA;
    if (persistent) t->flags |= NC_TF_PERSISTENT;
    return t;
}

nc_tensor *nc__tensor_alias(const nc_tensor *src, int persistent) {
    nc_tensor *t = (nc_tensor *)nc__meta_alloc(src->ctx, sizeof(nc_tensor), persistent);
    if (!t) return NULL;
    *t = *src;
    t->grad = NULL;
    t->node = NULL;
    t->name = NULL;
    t->owner = src->owner ? src->owner : (nc_tensor *)src;
    t->flags = persistent ? NC_TF_PERSISTENT : 0;
    t->host = NULL;
    t->coh = 0;
    t->bytes = 0;
    return t;
}

/* sets a fresh owner's contents from host bytes: upload + (small or asked) mirror */
static void fill_from_host(nc_tensor *t, const void *src, int keep_mirror) {
    nc_ctx *ctx = t->ctx;
    nc__upload(ctx, t->data, src, t->bytes);
    if (keep_mirror || t->bytes <= NC_MIRROR_SMALL) {
        void *h = mirror_of(t);
        if (h) {
            memcpy(h, src, t->bytes);
            t->coh = NC_COH_HOST_VALID;
        }
    }
}

nc_tensor *nc_empty(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape) {
    return nc__tensor_new(ctx, dt, ndim, shape, nc__is_persistent_mode(ctx));
}

nc_tensor *nc_zeros(nc_ctx *ctx, nc_dtype dt, int ndim, const int64_t *shape) {
    nc_tensor *t = nc_empty(ctx, dt, ndim, shape);
    if (!t) return NULL;
    nc__cuda_ok(ctx, cudaMemsetAsync(t->data, 0, t->bytes, (cudaStream_t)ctx->dev.stream), "memset");
    if (t->bytes <= NC_MIRROR_SMALL && mirror_of(t)) {
        memset(t->host, 0, t->bytes);
        t->coh = NC_COH_HOST_VALID;
    }
    return t;
}

nc_tensor *nc_full(nc_ctx *ctx, float value, int ndim, const int64_t *shape) {
    nc_tensor *t = nc_empty(ctx, NC_F32, ndim, shape);
    if (!t) return NULL;
    int64_t n = nc_numel(t);
    nck_fill_f32(nc__k(ctx), (float *)t->data, value, n);
    if (t->bytes <= NC_MIRROR_SMALL && mirror_of(t)) {
        for (int64_t i = 0; i < n; i++) ((float *)t->host)[i] = value;
        t->coh = NC_COH_HOST_VALID;
    }
    return t;
}

/* Random tensors are drawn on the host from the context's stream (bit-identical to newch's
 * nc_randn / nc_rand_uniform, engine/src/core/tensor.c:171-187) and uploaded. */
static nc_tensor *random_tensor(nc_ctx *ctx, int normal, float a, float b, int ndim, const int64_t *shape) {
    nc_tensor *t = nc_empty(ctx, NC_F32, ndim, shape);
    if (!t) return NULL;
    int64_t n = nc_numel(t);
    float *buf = (float *)malloc((size_t)(n ? n : 1) * sizeof(float));
    if (!buf) {
        nc__error(ctx, NC_ERR_OOM, "out of host memory");
        return NULL;
    }
    if (normal)
        for (int64_t i = 0; i < n; i++) buf[i] = a * nc__rand_normal(ctx);
    else
        for (int64_t i = 0; i < n; i++) buf[i] = a + (b - a) * nc__rand_uniform01(ctx);
    fill_from_host(t, buf, 0);
    free(buf);
    return t;
}

nc_tensor *nc_randn(nc_ctx *ctx, float stddev, int ndim, const int64_t *shape) {
    return random_tensor(ctx, 1, stddev, 0.0f, ndim, shape);
}

nc_tensor *nc_rand_uniform(nc_ctx *ctx, float lo, float hi, int ndim, const int64_t *shape) {
    return random_tensor(ctx, 0, lo, hi, ndim, shape);
}

nc_tensor *nc_from_data(nc_ctx *ctx, nc_dtype dt, const void *data, int ndim, const int64_t *shape) {
    nc_tensor *t = nc_empty(ctx, dt, ndim, shape);
    if (t && data) {
        /* integer tensors (labels, indices) keep their host copy: ops validate them without a
         * device round trip */
        int keep = (dt == NC_I32 || dt == NC_U8 || dt == NC_I8) && t->bytes <= ((size_t)1 << 20);
        fill_from_host(t, data, keep);
    }
    return t;
}

nc_tensor *nc_scalar(nc_ctx *ctx, float value) { return nc_full(ctx, value, 0, NULL); }

nc_tensor *nc_parameter(nc_ctx *ctx, const nc_tensor *init, int ndim, const int64_t *shape) {
    nc_tensor *t = nc__tensor_new(ctx, NC_F32, ndim, shape, 1);
    if (!t) return NULL;
    if (init) {
        if (init->dtype != NC_F32 || nc_numel(init) != nc_numel(t)) {
            nc__error(ctx, NC_ERR_SHAPE, "parameter init has %lld elements, expected %lld",
                      (long long)nc_numel(init), (long long)nc_numel(t));
            nc_release(t);
            return NULL;
        }
        nc_tensor *src = (nc_tensor *)init;
        const void *h = nc__host_view(src);
        if (h) {
            fill_from_host(t, h, 0);
        } else {
            nc__dev(src);
            nck_copy_strided(nc__k(ctx), 4, src->ndim, src->shape, src->stride, src->data, t->data);
        }
    } else {
        nc__cuda_ok(ctx, cudaMemsetAsync(t->data, 0, t->bytes, (cudaStream_t)ctx->dev.stream), "memset");
        if (t->bytes <= NC_MIRROR_SMALL && mirror_of(t)) {
            memset(t->host, 0, t->bytes);
            t->coh = NC_COH_HOST_VALID;
        }
    }
    t->flags |= NC_TF_REQUIRES_GRAD;
    return t;
}

/* ---- accessors -------------------------------------------------------------------------------- */

int nc_ndim(const nc_tensor *t) { return t ? t->ndim : 0; }
const int64_t *nc_shape(const nc_tensor *t) { return t ? t->shape : NULL; }
int64_t nc_numel(const nc_tensor *t) { return t ? nc__shape_numel(t->ndim, t->shape) : 0; }
nc_dtype nc_get_dtype(const nc_tensor *t) { return t ? t->dtype : NC_F32; }
int nc_requires_grad(const nc_tensor *t) { return t ? nc__needs_grad(t) : 0; }
nc_tensor *nc_grad(const nc_tensor *t) { return (t && !(t->flags & NC_TF_GRAD_CLEARED)) ? t->grad : NULL; }
int nc_is_persistent(const nc_tensor *t) { return t && (t->flags & NC_TF_PERSISTENT) != 0; }

void nc_release(nc_tensor *t) {
    if (!t || !(t->flags & NC_TF_PERSISTENT)) return;
    nc_ctx *ctx = t->ctx;
    if (t->grad) nc_release(t->grad);
    if (t->flags & NC_TF_OWNS_DATA) {
        nc__persistent_free(ctx, t->data, t->bytes);
        mirror_free(t);
    }
    free(t);
}

void nc_set_name(nc_tensor *t, const char *name) {
    if (t) t->name = name;
}
const char *nc_name(const nc_tensor *t) { return t && t->name ? t->name : ""; }

int64_t nc_dim(const nc_tensor *t, int axis) {
    if (!t) return 0;
    int a = nc__norm_axis(axis, t->ndim);
    return a < 0 ? 0 : t->shape[a];
}

void nc_set_requires_grad(nc_tensor *t, int on) {
    if (!t) return;
    if (on && t->dtype != NC_F32) {
        nc__error(t->ctx, NC_ERR_DTYPE, "only f32 tensors can require grad");
        return;
    }
    if (on) t->flags |= NC_TF_REQUIRES_GRAD;
    else t->flags &= ~NC_TF_REQUIRES_GRAD;
}

int nc_is_contiguous(const nc_tensor *t) {
    if (!t) return 0;
    int64_t s = 1;
    for (int i = t->ndim - 1; i >= 0; i--) {
        if (t->shape[i] != 1 && t->stride[i] != s) return 0;
        s *= t->shape[i];
    }
    return 1;
}

static void *data_host(nc_tensor *t, nc_dtype want) {
    if (!t || t->dtype != want || !nc_is_contiguous(t) || !t->data) return NULL;
    nc_tensor *o = nc__owner(t);
    char *h = (char *)mirror_refresh(o);
    if (!h) return NULL;
    o->coh |= NC_COH_HOST_DIRTY; /* the caller may write through it */
    return h + ((char *)t->data - (char *)o->data);
}

float *nc_data_f32(nc_tensor *t) { return (float *)data_host(t, NC_F32); }
int32_t *nc_data_i32(nc_tensor *t) { return (int32_t *)data_host(t, NC_I32); }

static float load_as_float(const void *p, nc_dtype dt) {
    switch (dt) {
    case NC_F32: return *(const float *)p;
    case NC_I32: return (float)*(const int32_t *)p;
    case NC_I8: return (float)*(const int8_t *)p;
    case NC_U8: return (float)*(const uint8_t *)p;
    default: return NAN;
    }
}

float nc_get(const nc_tensor *t, const int64_t *index) {
    if (!t || !t->data) return NAN;
    int64_t off = 0;
    for (int i = 0; i < t->ndim; i++) off += index[i] * t->stride[i];
    size_t es = nc__dtype_size(t->dtype);
    nc_tensor *o = nc__owner((nc_tensor *)t);
    const char *elem = (const char *)t->data + off * (int64_t)es;
    if ((o->coh & NC_COH_HOST_VALID) && o->host) return load_as_float((const char *)o->host + (elem - (const char *)o->data), t->dtype);
    unsigned char buf[8];
    nc__dev((nc_tensor *)t);
    nc__download(t->ctx, buf, elem, es);
    if (t->ctx->status != NC_OK) return NAN;
    return load_as_float(buf, t->dtype);
}

float nc_item(const nc_tensor *t) {
    if (!t || nc_numel(t) != 1) return NAN;
    int64_t zero[NC_MAX_DIMS] = {0};
    return nc_get(t, zero);
}

int nc_copy_to(const nc_tensor *t, void *dst, size_t dst_bytes) {
    if (!t || !dst) return 0;
    nc_ctx *ctx = t->ctx;
    size_t need = (size_t)nc_numel(t) * nc__dtype_size(t->dtype);
    if (dst_bytes < need) {
        nc__error(ctx, NC_ERR_ARG, "nc_copy_to: buffer has %zu bytes, need %zu", dst_bytes, need);
        return 0;
    }
    if (!need) return 1;
    nc_tensor *tt = (nc_tensor *)t;
    const void *h = nc__host_view(tt);
    if (h) {
        memcpy(dst, h, need);
        return 1;
    }
    const void *src = nc__contig(tt);
    if (!src) return 0;
    nc__download(ctx, dst, src, need);
    return ctx->status == NC_OK;
}

int nc_copy_from(nc_tensor *t, const void *src, size_t src_bytes) {
    if (!t || !src) return 0;
    size_t need = (size_t)nc_numel(t) * nc__dtype_size(t->dtype);
    if (!nc_is_contiguous(t) || src_bytes != need) {
        nc__error(t->ctx, NC_ERR_ARG, "nc_copy_from: need a contiguous tensor and exactly %zu bytes (got %zu)", need,
                  src_bytes);
        return 0;
    }
    nc_tensor *o = nc__owner(t);
    if (o->bytes <= NC_MIRROR_SMALL && !o->deferred && (need == o->bytes || (o->coh & NC_COH_HOST_VALID))) {
        /* a small owner (a scalar such as BatchNorm's batch counter): the bytes go to its host mirror,
         * marked as not yet on the device; the next device use uploads them (nc__dev), and a tensor
         * that only the host reads never pays a copy */
        char *h = (char *)mirror_of(o);
        if (h) {
            memcpy(h + ((char *)t->data - (char *)o->data), src, need);
            o->coh = NC_COH_HOST_VALID | NC_COH_HOST_DIRTY;
            return 1;
        }
    }
    nc__dev(t); /* earlier host writes must not land after this copy */
    nc__upload(t->ctx, t->data, src, need);
    if (o->host || o->bytes <= NC_MIRROR_SMALL) {
        char *h = (char *)mirror_of(o);
        if (h) {
            if (!(o->coh & NC_COH_HOST_VALID) && need != o->bytes) {
                o->coh = 0; /* partial write into a stale mirror: drop it */
            } else {
                memcpy(h + ((char *)t->data - (char *)o->data), src, need);
                o->coh = NC_COH_HOST_VALID;
            }
        }
    } else {
        o->coh &= ~NC_COH_HOST_VALID;
    }
    return 1;
}

/* ---- contiguous device views ------------------------------------------------------------------- */

const void *nc__contig(nc_tensor *t) {
    nc__dev(t);
    if (nc_is_contiguous(t)) return t->data;
    size_t es = nc__dtype_size(t->dtype);
    void *buf = nc__arena_alloc(t->ctx, (size_t)nc_numel(t) * es);
    if (buf) nck_copy_strided(nc__k(t->ctx), (int)es, t->ndim, t->shape, t->stride, t->data, buf);
    return buf;
}

const float *nc__contig_f32(nc_tensor *t) { return (const float *)nc__contig(t); }

nc_tensor *nc__grad_buf(nc_tensor *t) {
    nc_ctx *ctx = t->ctx;
    if (t->grad) nc__dev_write(t->grad); /* the caller accumulates into it on the device */
    if (t->grad && (t->flags & NC_TF_GRAD_CLEARED)) {
        nc__cuda_ok(ctx, cudaMemsetAsync(t->grad->data, 0, t->grad->bytes, (cudaStream_t)ctx->dev.stream), "memset");
        t->flags &= ~NC_TF_GRAD_CLEARED;
    }
    if (!t->grad) {
        int persistent = (t->flags & NC_TF_PERSISTENT) != 0;
        ctx->grad_alloc = 1;
        t->grad = nc__tensor_new(ctx, NC_F32, t->ndim, t->shape, persistent);
        ctx->grad_alloc = 0;
        if (t->grad)
            nc__cuda_ok(ctx, cudaMemsetAsync(t->grad->data, 0, t->grad->bytes, (cudaStream_t)ctx->dev.stream),
                        "memset");
    }
    return t->grad;
}

int nc__grad_handoff(nc_tensor *in, nc_tensor *out) {
    nc_tensor *g = out->grad;
    nc_ctx *ctx = in->ctx;
    if (!ctx->bwd_logging || !g || in->grad || (in->flags & NC_TF_PERSISTENT) || (g->flags & NC_TF_PERSISTENT) ||
        !(g->flags & NC_TF_OWNS_DATA) || in->dtype != NC_F32 || nc_numel(in) != nc_numel(g))
        return 0;
    nc__dev_write(g);
    g->ndim = in->ndim;
    memcpy(g->shape, in->shape, sizeof(int64_t) * (size_t)in->ndim);
    nc__contig_strides(in->ndim, g->shape, g->stride);
    in->grad = g;
    in->flags &= ~NC_TF_GRAD_CLEARED;
    out->grad = NULL;
    return 1;
}

nc_tensor *nc__grad_buf_acc(nc_tensor *t, int *acc) {
    *acc = 1;
    if (t->flags & NC_TF_PERSISTENT) return nc__grad_buf(t);
    nc_ctx *ctx = t->ctx;
    if (t->grad) {
        nc__dev_write(t->grad);
        if (t->flags & NC_TF_GRAD_CLEARED) {
            t->flags &= ~NC_TF_GRAD_CLEARED;
            *acc = 0;
        }
        return t->grad;
    }
    ctx->grad_alloc = 1;
    t->grad = nc__tensor_new(ctx, NC_F32, t->ndim, t->shape, 0);
    ctx->grad_alloc = 0;
    if (t->grad) *acc = 0;
    return t->grad;
}

/* ---- printing --------------------------------------------------------------------------------- */

void nc_print(const nc_tensor *t) {
    if (!t) {
        printf("tensor(NULL)\n");
        return;
    }
    printf("tensor(%s%s%s, %s, shape=[", t->name ? "\"" : "", t->name ? t->name : "", t->name ? "\"" : "",
           nc__dtype_name(t->dtype));
    for (int i = 0; i < t->ndim; i++) printf(i ? ", %lld" : "%lld", (long long)t->shape[i]);
    printf("]%s)\n  ", nc__needs_grad(t) ? ", grad" : "");
    int64_t n = nc_numel(t), shown = n < 32 ? n : 32;
    size_t es = nc__dtype_size(t->dtype);
    unsigned char *buf = (unsigned char *)malloc((size_t)(n ? n : 1) * es);
    if (buf && nc_copy_to(t, buf, (size_t)n * es)) {
        for (int64_t i = 0; i < shown; i++) printf("%.5g ", load_as_float(buf + i * (int64_t)es, t->dtype));
    }
    free(buf);
    printf(n > shown ? "... (%lld total)\n" : "\n", (long long)n);
}

/* ---- op registry ------------------------------------------------------------------------------ */

#define NC_OP_PTR(name) &nc_op_##name,
static const nc_op_def *const op_table[] = {NC_OP_LIST(NC_OP_PTR)};
#undef NC_OP_PTR

int nc__op_count(void) { return (int)(sizeof op_table / sizeof op_table[0]); }
const nc_op_def *nc__op_at(int i) { return (i >= 0 && i < nc__op_count()) ? op_table[i] : NULL; }
