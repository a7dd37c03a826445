/* Optimizers: SGD(+momentum), Adam, AdamW, RMSprop with gradient accumulation, one fused launch
 * per step for all parameters.
 *
 * Update rules, defaults, the accumulation gate and the state-slot layout are newch's
 * (engine/src/optim/optim.c: struct :15-27, create :29-67, defaults :81-104, accumulation :106-130,
 * state access :132-158, step :161-213, clip_grad_norm :216-233). What is B200-specific:
 *   - the optimizer owns one flat gradient buffer; every parameter's grad becomes a view into it,
 *     so data-parallel ranks all-reduce a single buffer (one NCCL call) before the update;
 *   - Adam's m and v are flat buffers too; one multi-segment kernel updates every parameter;
 *   - nc_optim_state hands out a host mirror of the flat state, uploaded again before the next step
 *     (newch/optim.py reads and writes it with ctypes.string_at / memmove).
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdlib.h>

enum { OPT_SGD = NCK_OPT_SGD, OPT_ADAM = NCK_OPT_ADAM, OPT_ADAMW = NCK_OPT_ADAMW, OPT_RMSPROP = NCK_OPT_RMSPROP };

struct nc_optim {
    nc_ctx *ctx;
    int kind;
    int n;
    nc_tensor **params;
    int64_t *off;      /* element offset of each parameter in the flat buffers */
    int64_t total;
    float *gflat;      /* device: all gradients */
    float *s1, *s2;    /* device: momentum / Adam m, Adam v / RMSprop square average (flat) */
    float *h1, *h2;    /* host mirrors of s1, s2 */
    int state_host_valid, state_host_dirty;
    nc_optim_opts o;
    int64_t t;
    int accum_steps, accum_count;
    int eps_inside_sqrt;
    nck_param_seg *segs;
};

/* The parameter's grad becomes a view into the flat buffer (keeping any gradient it holds). */
static int adopt_grad(nc_optim *opt, int i) {
    nc_ctx *ctx = opt->ctx;
    nc_tensor *p = opt->params[i];
    float *slot = opt->gflat + opt->off[i];
    size_t bytes = (size_t)nc_numel(p) * sizeof(float);
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    nc_tensor *g = (nc_tensor *)calloc(1, sizeof(nc_tensor));
    if (!g) return 0;
    g->ctx = ctx;
    g->dtype = NC_F32;
    g->ndim = p->ndim;
    memcpy(g->shape, p->shape, sizeof g->shape);
    nc__contig_strides(p->ndim, p->shape, g->stride);
    g->data = slot;
    g->bytes = bytes;
    g->flags = NC_TF_PERSISTENT; /* a view into the optimizer's buffer: nc_release frees the header only */
    if (p->grad) {
        nc__dev(p->grad);
        cudaMemcpyAsync(slot, p->grad->data, bytes, cudaMemcpyDeviceToDevice, s);
        nc_release(p->grad);
    } else {
        cudaMemsetAsync(slot, 0, bytes, s);
        p->flags |= NC_TF_GRAD_CLEARED; /* absent until a backward reaches it */
    }
    p->grad = g;
    return 1;
}

static nc_optim *create(nc_ctx *ctx, int kind, nc_tensor **params, int n, nc_optim_opts o) {
    for (int i = 0; i < n; i++) {
        nc_tensor *p = params[i];
        if (!p) return NULL;
        if (!(p->flags & NC_TF_PERSISTENT) || !nc__needs_grad(p) || p->dtype != NC_F32 || !nc_is_contiguous(p)) {
            nc__error(ctx, NC_ERR_ARG, "optimizer: param %d must be a contiguous f32 nc_parameter", i);
            return NULL;
        }
    }
    if (!ctx->device_ok) {
        nc__error(ctx, NC_ERR_STATE, "optimizer: no CUDA device");
        return NULL;
    }
    nc_optim *opt = (nc_optim *)calloc(1, sizeof(nc_optim));
    if (!opt) return NULL;
    opt->ctx = ctx;
    opt->kind = kind;
    opt->n = n;
    opt->o = o;
    opt->accum_steps = 1;
    opt->params = (nc_tensor **)calloc((size_t)(n ? n : 1), sizeof(nc_tensor *));
    opt->off = (int64_t *)calloc((size_t)(n ? n : 1), sizeof(int64_t));
    opt->segs = (nck_param_seg *)calloc((size_t)(n ? n : 1), sizeof(nck_param_seg));
    if (!opt->params || !opt->off || !opt->segs) goto fail;
    memcpy(opt->params, params, sizeof(nc_tensor *) * (size_t)n);
    for (int i = 0; i < n; i++) {
        opt->off[i] = opt->total;
        /* keep every parameter's slice 16-byte aligned for vector loads */
        opt->total += (nc_numel(params[i]) + 3) & ~(int64_t)3;
    }
    size_t bytes = (size_t)(opt->total ? opt->total : 1) * sizeof(float);
    int adam = kind == OPT_ADAM || kind == OPT_ADAMW;
    int need1 = adam || o.momentum != 0.0f, need2 = adam || kind == OPT_RMSPROP;
    opt->gflat = (float *)nc__persistent_alloc(ctx, bytes);
    if (!opt->gflat) goto fail;
    if (need1 && !(opt->s1 = (float *)nc__persistent_alloc(ctx, bytes))) goto fail;
    if (need2 && !(opt->s2 = (float *)nc__persistent_alloc(ctx, bytes))) goto fail;
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    if (opt->s1) cudaMemsetAsync(opt->s1, 0, bytes, s);
    if (opt->s2) cudaMemsetAsync(opt->s2, 0, bytes, s);
    for (int i = 0; i < n; i++)
        if (!adopt_grad(opt, i)) goto fail;
    opt->state_host_valid = 0;
    return opt;
fail:
    nc__error(ctx, NC_ERR_OOM, "optimizer: out of memory");
    nc_optim_free(opt);
    return NULL;
}

/* The parameters may already be gone when the optimizer is freed (Python drops objects in any
 * order at exit), so this touches only the optimizer's own state. The flat gradient buffer stays
 * allocated until nc_free_ctx: parameters that outlive the optimizer keep their grads. */
void nc_optim_free(nc_optim *o) {
    if (!o) return;
    nc_ctx *ctx = o->ctx;
    size_t bytes = (size_t)(o->total ? o->total : 1) * sizeof(float);
    if (o->s1) nc__persistent_free(ctx, o->s1, bytes);
    if (o->s2) nc__persistent_free(ctx, o->s2, bytes);
    if (o->h1) cudaFreeHost(o->h1);
    if (o->h2) cudaFreeHost(o->h2);
    free(o->params);
    free(o->off);
    free(o->segs);
    free(o);
}

nc_optim *nc_sgd(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts) {
    return create(ctx, OPT_SGD, params, n, opts);
}

static nc_optim_opts adam_defaults(nc_optim_opts opts) {
    if (opts.beta1 == 0.0f) opts.beta1 = 0.9f;
    if (opts.beta2 == 0.0f) opts.beta2 = 0.999f;
    if (opts.eps == 0.0f) opts.eps = 1e-8f;
    return opts;
}

nc_optim *nc_adam(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts) {
    return create(ctx, OPT_ADAM, params, n, adam_defaults(opts));
}

nc_optim *nc_adamw(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts) {
    return create(ctx, OPT_ADAMW, params, n, adam_defaults(opts));
}

nc_optim *nc_rmsprop(nc_ctx *ctx, nc_tensor **params, int n, nc_optim_opts opts, int eps_inside_sqrt) {
    if (opts.beta2 == 0.0f) opts.beta2 = 0.99f;
    if (opts.eps == 0.0f) opts.eps = 1e-8f;
    nc_optim *o = create(ctx, OPT_RMSPROP, params, n, opts);
    if (o) o->eps_inside_sqrt = eps_inside_sqrt ? 1 : 0;
    return o;
}

void nc_optim_set_accumulation(nc_optim *o, int steps) {
    if (!o) return;
    if (steps < 1) {
        nc__error(o->ctx, NC_ERR_ARG, "gradient accumulation steps must be >= 1, got %d", steps);
        return;
    }
    o->accum_steps = steps;
    o->accum_count = 0;
}

void nc_optim_zero_grad(nc_optim *o) {
    if (!o || o->accum_count != 0) return;
    for (int i = 0; i < o->n; i++) nc_zero_grad(o->params[i]);
}

void nc_optim_clear_grad(nc_optim *o) {
    if (!o || o->accum_count != 0) return;
    for (int i = 0; i < o->n; i++) nc_clear_grad(o->params[i]);
}

void nc_optim_set_lr(nc_optim *o, float lr) {
    if (o) o->o.lr = lr;
}

static void state_upload_if_dirty(nc_optim *o) {
    if (!o->state_host_dirty) return;
    size_t bytes = (size_t)o->total * sizeof(float);
    if (o->s1 && o->h1) nc__upload(o->ctx, o->s1, o->h1, bytes);
    if (o->s2 && o->h2) nc__upload(o->ctx, o->s2, o->h2, bytes);
    o->state_host_dirty = 0;
}

float *nc_optim_state(nc_optim *o, int param, int slot) {
    if (!o || param < 0 || param >= o->n || slot < 0 || slot > 1) return NULL;
    float *dev = slot == 0 ? o->s1 : o->s2;
    if (!dev) return NULL;
    if (!o->state_host_valid) {
        size_t bytes = (size_t)(o->total ? o->total : 1) * sizeof(float);
        if (o->s1 && !o->h1 && cudaMallocHost((void **)&o->h1, bytes) != cudaSuccess) return NULL;
        if (o->s2 && !o->h2 && cudaMallocHost((void **)&o->h2, bytes) != cudaSuccess) return NULL;
        state_upload_if_dirty(o);
        if (o->s1) nc__download(o->ctx, o->h1, o->s1, (size_t)o->total * sizeof(float));
        if (o->s2) nc__download(o->ctx, o->h2, o->s2, (size_t)o->total * sizeof(float));
        if (o->ctx->status != NC_OK) return NULL;
        o->state_host_valid = 1;
    }
    o->state_host_dirty = 1;
    return (slot == 0 ? o->h1 : o->h2) + o->off[param];
}

int64_t nc_optim_get_step(const nc_optim *o) { return o ? o->t : 0; }

void nc_optim_set_step(nc_optim *o, int64_t t) {
    if (!o) return;
    if (t < 0) {
        nc__error(o->ctx, NC_ERR_ARG, "optimizer step count must be >= 0, got %lld", (long long)t);
        return;
    }
    o->t = t;
    o->accum_count = 0;
}

void nc_optim_set_opts(nc_optim *o, nc_optim_opts opts) {
    if (!o) return;
    int adam = o->kind == OPT_ADAM || o->kind == OPT_ADAMW;
    int has_momentum = !adam && o->s1 != NULL;
    if (!adam && has_momentum != (opts.momentum != 0.0f)) {
        nc__error(o->ctx, NC_ERR_ARG, "optimizer: momentum cannot switch between zero and non-zero (%g -> %g)",
                  (double)o->o.momentum, (double)opts.momentum);
        return;
    }
    o->o = opts;
}

void nc_optim_step(nc_optim *o) {
    if (!o || !nc_ok(o->ctx)) return;
    if (o->accum_steps > 1 && ++o->accum_count < o->accum_steps) return;
    o->accum_count = 0;
    nc_ctx *ctx = o->ctx;
    const nc_optim_opts *c = &o->o;
    nck_opt_hyper h;
    memset(&h, 0, sizeof h);
    h.kind = o->kind;
    h.lr = c->lr, h.momentum = c->momentum, h.weight_decay = c->weight_decay;
    h.beta1 = c->beta1, h.beta2 = c->beta2, h.eps = c->eps;
    h.gs = 1.0f / (float)o->accum_steps;
    h.eps_inside_sqrt = o->eps_inside_sqrt;
    o->t++;
    h.bc1 = 1.0f, h.bc2 = 1.0f;
    if (o->kind == OPT_ADAM || o->kind == OPT_ADAMW) {
        h.bc1 = 1.0f - powf(c->beta1, (float)o->t);
        h.bc2 = 1.0f - powf(c->beta2, (float)o->t);
    }
    state_upload_if_dirty(o);
    if (ctx->dp_world > 1) {
        /* absent gradients count as zero in the sum over ranks */
        for (int i = 0; i < o->n; i++)
            if (!nc_grad(o->params[i]) && o->params[i]->grad)
                cudaMemsetAsync(o->params[i]->grad->data, 0, o->params[i]->grad->bytes, (cudaStream_t)ctx->dev.stream);
        for (int i = 0; i < o->n; i++)
            if (o->params[i]->grad) nc__dev(o->params[i]->grad);
        if (!nc__dp_allreduce_mean(ctx, o->gflat, o->total)) return;
    }
    int nseg = 0;
    for (int i = 0; i < o->n; i++) {
        nc_tensor *p = o->params[i];
        nc_tensor *gt = nc_grad(p);
        if (!gt && ctx->dp_world <= 1) continue;
        if (!gt && !p->grad) continue;
        if (!gt) gt = p->grad;
        nc__dev_write(p);
        nck_param_seg *sg = &o->segs[nseg++];
        sg->w = (float *)nc__dev(p);
        sg->g = (const float *)nc__dev(gt);
        sg->m = o->s1 ? o->s1 + o->off[i] : NULL;
        sg->v = o->s2 ? o->s2 + o->off[i] : NULL;
        sg->n = nc_numel(p);
    }
    if (nseg) nck_optim_step(nc__k(ctx), &h, o->segs, nseg);
    o->state_host_valid = 0;
}

float nc_clip_grad_norm(nc_tensor **params, int n, float max_norm) {
    nc_ctx *ctx = NULL;
    for (int i = 0; i < n && !ctx; i++)
        if (params[i]) ctx = params[i]->ctx;
    if (!ctx || !ctx->device_ok) return 0.0f;
    double *acc = (double *)nc__arena_alloc(ctx, sizeof(double));
    if (!acc) return 0.0f;
    int first = 1;
    for (int i = 0; i < n; i++) {
        nc_tensor *g = params[i] ? nc_grad(params[i]) : NULL;
        if (!g) continue;
        nck_sumsq(nc__k(ctx), (const float *)nc__dev(g), nc_numel(g), acc, !first);
        first = 0;
    }
    double ss = 0.0;
    if (!first) nc__download(ctx, &ss, acc, sizeof ss);
    float total = (float)sqrt(ss);
    float coef = max_norm / (total + 1e-6f);
    if (coef < 1.0f) {
        for (int i = 0; i < n; i++) {
            nc_tensor *g = params[i] ? nc_grad(params[i]) : NULL;
            if (!g) continue;
            nc__dev_write(g);
            nck_unary_fwd(nc__k(ctx), NCK_UN_SCALE, coef, (const float *)g->data, (float *)g->data, nc_numel(g));
        }
    }
    return total;
}
