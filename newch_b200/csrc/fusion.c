/* Deferred epilogues and fused backward chains around BatchNorm.
 *
 * newch's models apply BatchNorm, then an activation, then often a 2 x 2 max pool, as three ops each
 * reading and writing a full activation tensor. This engine keeps their results (and gradients)
 * identical while moving far less data:
 *
 *   forward   BatchNorm in training computes only its statistics; its output becomes a recipe
 *             (x and the per-channel affine). A following piecewise activation extends the recipe.
 *             A 2 x 2 / stride 2 max pool over a recipe pools straight from x (one pass writing the
 *             quarter-size output and its argmax). Any other reader materialises the recipe with one
 *             normalise-and-activate pass (nc__dev, the host paths).
 *   backward  when the pool's input and the BatchNorm output still hold recipes (nothing else read
 *             them) and each has a single consumer in the pass, the pool's backward runs the chain
 *             as one BatchNorm backward fed with the sparse pooled gradient; an activation over a
 *             BatchNorm output likewise folds into the BatchNorm backward. The intermediate
 *             gradients are never formed.
 *
 * Values are the unfused ones: the recipe is evaluated with the normalisation kernel's arithmetic
 * (x * a + d with a = w * invstd, d = b - mean * a, then the activation in newch's formula), and the
 * fused backward forms the same per-element gradient before the same BatchNorm reductions.
 * NC_FUSE=0 turns all of it off.
 */
#include "nc_internal.h"

void nc__defer_bn(nc_ctx *ctx, nc_tensor *out, nc_tensor *x, const float *X, const float *w, const float *b,
                  const float *mean, const float *invstd, int64_t N, int64_t C, int64_t S) {
    nc_deferred *d = (nc_deferred *)nc__meta_alloc(ctx, sizeof(nc_deferred), 0);
    if (!d) return; /* out of host memory: nc__meta_alloc set the error */
    d->owner = out, d->src = nc__owner(x);
    d->x = X, d->w = w, d->b = b, d->mean = mean, d->invstd = invstd;
    d->N = N, d->C = C, d->S = S, d->act = -1, d->act_s = 0.0f;
    d->next = ctx->deferred_head;
    ctx->deferred_head = d;
    out->deferred = d;
}

const nc_deferred *nc__deferred_of(const nc_tensor *t) {
    if (!t || t->owner || !t->deferred) return NULL;
    return t->deferred;
}

int nc__defer_act(nc_tensor *out, nc_tensor *t, int act, float act_s) {
    const nc_deferred *src = nc__deferred_of(t);
    if (!src || src->act >= 0 || !nck_epi_supported(act) || act < 0) return 0;
    nc_ctx *ctx = t->ctx;
    nc_deferred *d = (nc_deferred *)nc__meta_alloc(ctx, sizeof(nc_deferred), 0);
    if (!d) return 0;
    *d = *src;
    d->owner = out, d->act = act, d->act_s = act_s;
    d->next = ctx->deferred_head;
    ctx->deferred_head = d;
    out->deferred = d;
    return 1;
}

static void unlink_deferred(nc_ctx *ctx, nc_deferred *d) {
    for (nc_deferred **p = &ctx->deferred_head; *p; p = &(*p)->next)
        if (*p == d) {
            *p = d->next;
            break;
        }
    d->owner->deferred = NULL;
}

void nc__materialize(nc_tensor *owner) {
    nc_deferred *d = owner->deferred;
    if (!d) return;
    nc_ctx *ctx = owner->ctx;
    unlink_deferred(ctx, d); /* first: the launch below reads no recipe */
    nck_bn_apply(nc__k(ctx), d->x, d->w, d->b, d->mean, d->invstd, (float *)owner->data, d->N, d->C, d->S, d->act,
                 d->act_s);
}

void nc__deferred_release(nc_tensor *owner) {
    nc_ctx *ctx = owner->ctx;
    if (!ctx->deferred_head) return;
    for (nc_deferred *d = ctx->deferred_head, *next; d; d = next) {
        next = d->next;
        if (d->src == owner && d->owner != owner) nc__materialize(d->owner);
    }
    if (owner->deferred) unlink_deferred(ctx, owner->deferred);
}

void nc__deferred_flush(nc_ctx *ctx) {
    while (ctx->deferred_head) nc__materialize(ctx->deferred_head->owner);
}

void nc__deferred_reset(nc_ctx *ctx) {
    for (nc_deferred *d = ctx->deferred_head; d; d = d->next) d->owner->deferred = NULL;
    ctx->deferred_head = NULL;
}

/* ---- fused backward chains ---------------------------------------------------------------------- */

/* t is an intermediate whose only consumer in this pass is one node and whose values were never read */
static int private_recipe(const nc_tensor *t, uint32_t epoch) {
    return nc__deferred_of(t) && t->use_epoch == epoch && t->uses == 1 && t->node;
}

static int is_bn_training(const nc_node *n) { return n->op == &nc_op_batch_norm && n->p.i[0] == 1; }

/* BatchNorm's saved statistics (ops_nn.c keeps them as {mean, invstd}) */
typedef struct {
    float *mean, *invstd;
} bn_saved_view;

static int bn_chain_args(nc_node *nb, const float **x, const float **w, const float **b, const bn_saved_view **sv) {
    nc_tensor *xt = nb->in[0];
    if (!nc_is_contiguous(xt) || !nb->saved) return 0;
    *x = (const float *)nc__dev(xt);
    *w = (const float *)nc__dev(nb->in[1]);
    *b = (const float *)nc__dev(nb->in[2]);
    *sv = (const bn_saved_view *)nb->saved;
    return 1;
}

/* the BatchNorm input's and parameters' gradient buffers, as BatchNorm's own backward takes them */
static void bn_grads(nc_node *nb, float **gx, int *acc_gx, float **gw, float **gb) {
    nc_tensor *x = nb->in[0], *w = nb->in[1], *b = nb->in[2];
    *acc_gx = 1;
    nc_tensor *tx = nc__needs_grad(x) ? nc__grad_buf_acc(x, acc_gx) : NULL;
    nc_tensor *tw = nc__needs_grad(w) ? nc__grad_buf(w) : NULL;
    nc_tensor *tb = nc__needs_grad(b) ? nc__grad_buf(b) : NULL;
    *gx = tx ? (float *)tx->data : NULL;
    *gw = tw ? (float *)tw->data : NULL;
    *gb = tb ? (float *)tb->data : NULL;
}

static void bn_dims(const nc_tensor *x, int64_t *N, int64_t *C, int64_t *S) {
    *N = x->shape[0];
    *C = x->ndim > 1 ? x->shape[1] : 1;
    *S = 1;
    for (int i = 2; i < x->ndim; i++) *S *= x->shape[i];
}

/* max pool 2 x 2, stride 2, no padding over an (act of a) BatchNorm output */
static int fuse_pool_chain(nc_ctx *ctx, nc_node *np, nc_node **consumed) {
    if (np->op != &nc_op_max_pool2d || !np->saved) return 0;
    const int64_t *p = np->p.i; /* sh, sw, ph, pw, kh, kw */
    if (p[0] != 2 || p[1] != 2 || p[2] != 0 || p[3] != 0 || p[4] != 2 || p[5] != 2) return 0;
    const uint32_t ep = ctx->mark_epoch;
    nc_tensor *z = np->in[0];
    if (!private_recipe(z, ep)) return 0;
    const nc_deferred *rz = z->deferred;
    nc_node *na = NULL, *nb = z->node;
    if (rz->act >= 0) {
        na = z->node;
        if (nc__unary_kind(na->op) != rz->act || na->fused == ep) return 0;
        nc_tensor *y = na->in[0];
        if (!private_recipe(y, ep) || y->deferred->act >= 0) return 0;
        nb = y->node;
    }
    if (!is_bn_training(nb) || nb->fused == ep || z->ndim != 4) return 0;
    nc_tensor *x = nb->in[0];
    if (!nck_bn_pool2x2_ok(x->shape[0], x->shape[1], x->shape[2], x->shape[3])) return 0;
    const float *X, *w, *b;
    const bn_saved_view *sv;
    if (!bn_chain_args(nb, &X, &w, &b, &sv)) return 0;
    float *gx, *gw, *gb;
    int acc;
    bn_grads(nb, &gx, &acc, &gw, &gb);
    nck_bn_pool_bwd(nc__k(ctx), X, w, b, (const float *)np->out->grad->data, (const int32_t *)np->saved, sv->mean,
                    sv->invstd, gx, gw, gb, x->shape[0], x->shape[1], x->shape[2], x->shape[3], acc, rz->act,
                    rz->act_s);
    int k = 0;
    if (na) consumed[k++] = na;
    consumed[k++] = nb;
    return k;
}

/* a piecewise activation over a BatchNorm output */
static int fuse_act_chain(nc_ctx *ctx, nc_node *na, nc_node **consumed) {
    const int kind = nc__unary_kind(na->op);
    if (kind < 0 || !nck_epi_supported(kind)) return 0;
    const uint32_t ep = ctx->mark_epoch;
    nc_tensor *y = na->in[0];
    if (!private_recipe(y, ep) || y->deferred->act >= 0) return 0;
    nc_node *nb = y->node;
    if (!is_bn_training(nb) || nb->fused == ep) return 0;
    nc_tensor *x = nb->in[0];
    const float *X, *w, *b;
    const bn_saved_view *sv;
    if (!bn_chain_args(nb, &X, &w, &b, &sv)) return 0;
    float *gx, *gw, *gb;
    int acc;
    bn_grads(nb, &gx, &acc, &gw, &gb);
    int64_t N, C, S;
    bn_dims(x, &N, &C, &S);
    nck_bn_bwd_ex(nc__k(ctx), X, w, b, (const float *)na->out->grad->data, sv->mean, sv->invstd, gx, gw, gb, N, C, S,
                  1, acc, kind, na->p.f[0]);
    consumed[0] = nb;
    return 1;
}

int nc__fused_backward(nc_ctx *ctx, nc_node *n, nc_node **consumed) {
    if (!ctx->fuse || !n->out->grad) return 0;
    int k = fuse_pool_chain(ctx, n, consumed);
    if (!k) k = fuse_act_chain(ctx, n, consumed);
    return k;
}
