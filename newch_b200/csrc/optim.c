/* Optimizers: SGD(+momentum), Adam, AdamW, RMSprop with gradient accumulation, one fused launch
 * per step for all parameters.
 *
 * Update rules, defaults, the accumulation gate and the state-slot layout are newch's
 * (engine/src/optim/optim.c: struct :15-27, create :29-67, defaults :81-104, accumulation :106-130,
 * state access :132-158, step :161-213, clip_grad_norm :216-233). What is B200-specific:
 *   - the optimizer owns one flat gradient buffer; every parameter's grad becomes a view into it;
 *   - Adam's m and v are flat buffers too; one launch updates every parameter, each block one
 *     chunk of one parameter (a table built once and kept on the device);
 *   - nc_optim_state hands out a host mirror of the flat state, uploaded again before the next step
 *     (newch/optim.py reads and writes it with ctypes.string_at / memmove);
 *   - data parallelism: the flat buffer is cut into buckets of consecutive parameters (about 1 MiB,
 *     filled from the last parameter, whose gradient a backward pass finishes first). When a
 *     backward pass has enqueued the last writer of every parameter of a bucket, the bucket's mean
 *     over ranks is enqueued on the communication stream into a second flat buffer, so the
 *     all-reduces overlap the rest of the pass; the step reduces what is left, joins, and updates
 *     from the reduced buffer. A parameter with no gradient on any rank (a presence byte per
 *     parameter, maximum over ranks) is skipped as a single-GPU run skips it; one absent on some
 *     ranks only counts as zero there.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdlib.h>

enum { OPT_SGD = NCK_OPT_SGD, OPT_ADAM = NCK_OPT_ADAM, OPT_ADAMW = NCK_OPT_ADAMW, OPT_RMSPROP = NCK_OPT_RMSPROP };

typedef struct {
    int p0, p1;      /* parameters [p0, p1) */
    int64_t e0, e1;  /* their elements in the flat buffers */
    int expect;      /* parameters of the bucket the running backward pass has still to finish */
    int touched;     /* the running pass writes at least one of them */
    int fresh;       /* gred holds the mean over ranks of the bucket's current gradients */
} grad_bucket;

#define NC_BUCKET_FLOATS ((int64_t)1 << 18) /* 1 MiB */

struct nc_optim {
    nc_ctx *ctx;
    nc_optim *next_in_ctx;
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
    /* update launch: segments and chunks on the host (last built) and on the device */
    nck_param_seg *segs, *dsegs;
    nck_opt_chunk *chunks, *dchunks;
    int nseg, nchunk, cap_chunk;
    /* data parallel */
    float *gred;             /* device: gradients averaged over ranks */
    grad_bucket *bk;
    int nbk;
    int *bucket_of;          /* bucket of each parameter */
    unsigned char *pres_h, *pres_d; /* presence bytes (host staging / device, max over ranks) */
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
    p->optim = opt;
    p->optim_slot = i;
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
    opt->segs = (nck_param_seg *)calloc((size_t)(n ? 2 * n : 2), sizeof(nck_param_seg)); /* built | scratch */
    opt->nseg = -1; /* no table built yet */
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
    opt->next_in_ctx = ctx->optims;
    ctx->optims = opt;
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
    for (nc_optim **link = &ctx->optims; *link; link = &(*link)->next_in_ctx)
        if (*link == o) {
            *link = o->next_in_ctx;
            break;
        }
    nc__dp_join(ctx);
    if (ctx->device_ok) cudaStreamSynchronize((cudaStream_t)ctx->dev.stream);
    size_t bytes = (size_t)(o->total ? o->total : 1) * sizeof(float);
    if (o->s1) nc__persistent_free(ctx, o->s1, bytes);
    if (o->s2) nc__persistent_free(ctx, o->s2, bytes);
    if (o->gred) nc__persistent_free(ctx, o->gred, bytes);
    if (o->dsegs) nc__persistent_free(ctx, o->dsegs, sizeof(nck_param_seg) * (size_t)(o->n ? o->n : 1));
    if (o->dchunks) nc__persistent_free(ctx, o->dchunks, sizeof(nck_opt_chunk) * (size_t)o->cap_chunk);
    if (o->pres_d) nc__persistent_free(ctx, o->pres_d, (size_t)(o->n ? o->n : 1));
    if (o->h1) cudaFreeHost(o->h1);
    if (o->h2) cudaFreeHost(o->h2);
    free(o->params);
    free(o->off);
    free(o->segs);
    free(o->chunks);
    free(o->bk);
    free(o->bucket_of);
    free(o->pres_h);
    free(o);
}

/* ---- data-parallel gradient buckets ------------------------------------------------------------- */

/* o when it is still one of its context's optimizers (a parameter can outlive its optimizer) */
static nc_optim *live_optim(nc_tensor *p) {
    nc_optim *o = p->optim;
    if (!o) return NULL;
    for (nc_optim *q = p->ctx->optims; q; q = q->next_in_ctx)
        if (q == o) return (p->optim_slot >= 0 && p->optim_slot < o->n && o->params[p->optim_slot] == p) ? o : NULL;
    return NULL;
}

/* Buckets, the reduced buffer and the presence bytes, made when the context first runs data
 * parallel. Returns 1 when the optimizer all-reduces. */
static int dp_ready(nc_optim *o) {
    nc_ctx *ctx = o->ctx;
    if (ctx->dp_world <= 1) return 0;
    if (o->bk) return 1;
    size_t bytes = (size_t)(o->total ? o->total : 1) * sizeof(float);
    o->gred = (float *)nc__persistent_alloc(ctx, bytes);
    o->bk = (grad_bucket *)calloc((size_t)(o->n ? o->n : 1), sizeof(grad_bucket));
    o->bucket_of = (int *)calloc((size_t)(o->n ? o->n : 1), sizeof(int));
    o->pres_h = (unsigned char *)calloc((size_t)(o->n ? o->n : 1), 1);
    o->pres_d = (unsigned char *)nc__persistent_alloc(ctx, (size_t)(o->n ? o->n : 1));
    if (!o->gred || !o->bk || !o->bucket_of || !o->pres_h || !o->pres_d) {
        nc__error(ctx, NC_ERR_OOM, "optimizer: out of memory for data-parallel buffers");
        return 0;
    }
    /* from the last parameter backwards: a bucket closes once it holds NC_BUCKET_FLOATS */
    int nb = 0;
    for (int hi = o->n; hi > 0;) {
        int lo = hi;
        int64_t sz = 0;
        while (lo > 0 && (sz == 0 || sz + (o->off[lo] - o->off[lo - 1]) <= NC_BUCKET_FLOATS)) {
            lo--;
            sz = o->off[hi - 1] + ((nc_numel(o->params[hi - 1]) + 3) & ~(int64_t)3) - o->off[lo];
        }
        grad_bucket *b = &o->bk[nb];
        b->p0 = lo, b->p1 = hi;
        b->e0 = o->off[lo];
        b->e1 = o->off[hi - 1] + ((nc_numel(o->params[hi - 1]) + 3) & ~(int64_t)3);
        for (int i = lo; i < hi; i++) o->bucket_of[i] = nb;
        nb++;
        hi = lo;
    }
    o->nbk = nb;
    return 1;
}

/* Enqueues the bucket's all-reduce. Parameters whose gradient was cleared (set_to_none) and not
 * written since hold last cycle's values in their slots: they count as zero. */
static void launch_bucket(nc_optim *o, grad_bucket *b) {
    nc_ctx *ctx = o->ctx;
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    for (int i = b->p0; i < b->p1; i++) {
        nc_tensor *p = o->params[i];
        if (!nc_grad(p) && p->grad) cudaMemsetAsync(p->grad->data, 0, p->grad->bytes, s);
        else if (p->grad) nc__dev(p->grad); /* host writes to a gradient reach the device first */
    }
    if (nc__dp_reduce_async(ctx, o->gflat + b->e0, o->gred + b->e0, b->e1 - b->e0)) b->fresh = 1;
}

void nc__grad_pass_begin(nc_ctx *ctx) {
    if (!ctx->optims) return;
    nc__dp_join(ctx); /* reduces still reading the gradients this pass is about to write */
    for (nc_optim *o = ctx->optims; o; o = o->next_in_ctx)
        for (int b = 0; b < o->nbk; b++) o->bk[b].expect = o->bk[b].touched = 0;
}

void nc__grad_expect(nc_tensor *leaf) {
    nc_optim *o = live_optim(leaf);
    if (!o || !dp_ready(o)) return;
    grad_bucket *b = &o->bk[o->bucket_of[leaf->optim_slot]];
    b->expect++;
    b->touched = 1;
    b->fresh = 0;
}

void nc__grad_final(nc_tensor *leaf) {
    nc_optim *o = live_optim(leaf);
    if (!o || !o->bk) return;
    grad_bucket *b = &o->bk[o->bucket_of[leaf->optim_slot]];
    if (b->expect > 0 && --b->expect == 0 && o->accum_steps == 1) launch_bucket(o, b);
}

static void mark_stale(nc_optim *o) {
    for (int b = 0; b < o->nbk; b++) o->bk[b].fresh = 0;
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
    nc__dp_join(o->ctx);
    mark_stale(o);
    /* the gradients are views into one flat buffer: one memset clears them all (a memset per
     * parameter is a GPU operation each, ~50 per step for a transformer) */
    int flat = o->gflat != NULL && o->total > 0;
    for (int i = 0; i < o->n && flat; i++) {
        nc_tensor *p = o->params[i];
        flat = p->grad && p->grad->data == (void *)(o->gflat + o->off[i]);
    }
    if (!flat) {
        for (int i = 0; i < o->n; i++) nc_zero_grad(o->params[i]);
        return;
    }
    for (int i = 0; i < o->n; i++) {
        nc_tensor *p = o->params[i];
        if (!(p->flags & NC_TF_GRAD_CLEARED)) nc__dev_write(p->grad); /* pending host writes land first */
    }
    /* a cleared (absent) gradient's slot is zeroed too, which it is whenever it is next used */
    nc__cuda_ok(o->ctx, cudaMemsetAsync(o->gflat, 0, (size_t)o->total * sizeof(float), (cudaStream_t)o->ctx->dev.stream),
                "memset");
}

void nc_optim_clear_grad(nc_optim *o) {
    if (!o || o->accum_count != 0) return;
    mark_stale(o);
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

/* The update launch's tables on the device, rebuilt and uploaded only when the list of segments
 * differs from the one uploaded last (normally once, at the first step). */
static int upload_tables(nc_optim *o, const nck_param_seg *segs, int nseg) {
    nc_ctx *ctx = o->ctx;
    if (o->nseg == nseg && o->dsegs && !memcmp(o->segs, segs, sizeof(nck_param_seg) * (size_t)nseg)) return 1;
    if (!o->dsegs && !(o->dsegs = (nck_param_seg *)nc__persistent_alloc(ctx, sizeof(nck_param_seg) *
                                                                                (size_t)(o->n ? o->n : 1))))
        return 0;
    int nchunk = nck_optim_chunks(segs, nseg, NULL);
    if (nchunk > o->cap_chunk) {
        if (o->dchunks) nc__persistent_free(ctx, o->dchunks, sizeof(nck_opt_chunk) * (size_t)o->cap_chunk);
        free(o->chunks);
        o->cap_chunk = 0;
        o->chunks = (nck_opt_chunk *)malloc(sizeof(nck_opt_chunk) * (size_t)nchunk);
        o->dchunks = (nck_opt_chunk *)nc__persistent_alloc(ctx, sizeof(nck_opt_chunk) * (size_t)nchunk);
        if (!o->chunks || !o->dchunks) return 0;
        o->cap_chunk = nchunk;
    }
    nck_optim_chunks(segs, nseg, o->chunks);
    if (segs != o->segs) memcpy(o->segs, segs, sizeof(nck_param_seg) * (size_t)nseg);
    nc__upload(ctx, o->dsegs, o->segs, sizeof(nck_param_seg) * (size_t)nseg);
    nc__upload(ctx, o->dchunks, o->chunks, sizeof(nck_opt_chunk) * (size_t)nchunk);
    o->nseg = nseg;
    o->nchunk = nchunk;
    return ctx->status == NC_OK;
}

/* Data parallel: every bucket not reduced since its last write is reduced now (the same calls on
 * every rank, which all run the same graph), then the presence bytes, then the main stream waits. */
static int dp_finish_reduce(nc_optim *o) {
    nc_ctx *ctx = o->ctx;
    for (int b = 0; b < o->nbk; b++)
        if (!o->bk[b].fresh) launch_bucket(o, &o->bk[b]);
    if (ctx->bn_n && !nc__dp_bn_flush(ctx, 1)) return 0;
    for (int i = 0; i < o->n; i++) o->pres_h[i] = nc_grad(o->params[i]) ? 1 : 0;
    nc__upload(ctx, o->pres_d, o->pres_h, (size_t)o->n);
    if (!nc__dp_max_bytes_async(ctx, o->pres_d, o->n)) return 0;
    nc__dp_join(ctx);
    for (int b = 0; b < o->nbk; b++) o->bk[b].fresh = 0; /* the next cycle writes new gradients */
    return ctx->status == NC_OK;
}

void nc_optim_step(nc_optim *o) {
    if (!o || !nc_ok(o->ctx)) return;
    nc__deferred_flush(o->ctx); /* pending recipes read the parameters this step changes */
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
    const int dp = dp_ready(o);
    if (ctx->status != NC_OK || (dp && !dp_finish_reduce(o))) return;
    /* segments: parameters with a gradient here; under data parallelism every parameter, gated on
     * the device by whether any rank had its gradient */
    nck_param_seg *segs = o->segs + o->n; /* scratch half of the array */
    int nseg = 0;
    int64_t total = 0;
    for (int i = 0; i < o->n; i++) {
        nc_tensor *p = o->params[i];
        nc_tensor *gt = nc_grad(p);
        if (!gt && !dp) continue;
        if (gt) nc__dev(gt);
        nc__dev_write(p);
        nck_param_seg *sg = &segs[nseg++];
        memset(sg, 0, sizeof *sg);
        sg->w = (float *)nc__dev(p);
        sg->g = (dp ? o->gred : o->gflat) + o->off[i];
        sg->m = o->s1 ? o->s1 + o->off[i] : NULL;
        sg->v = o->s2 ? o->s2 + o->off[i] : NULL;
        sg->n = nc_numel(p);
        sg->param = i;
        total += sg->n;
    }
    if (nseg && upload_tables(o, segs, nseg))
        nck_optim_step(nc__k(ctx), &h, o->dsegs, o->dchunks, o->nchunk, total, dp ? o->pres_d : NULL);
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
