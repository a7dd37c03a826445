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
    memset(d, 0, sizeof *d);
    d->owner = out, d->src[0] = nc__owner(x), d->kind = NC_DEF_BN;
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
    if (!src || src->kind != NC_DEF_BN || src->act >= 0 || !nck_epi_supported(act) || act < 0) return 0;
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

/* an adopted source block goes back to the arena (after the last launch that reads it is enqueued) */
static void free_adopted(nc_ctx *ctx, nc_deferred *d) {
    if (!d->adopt) return;
    nc__arena_free(ctx, d->adopt, d->adopt_bytes);
    d->adopt = NULL;
}

int nc__deferred_adopt(nc_tensor *owner) {
    nc_ctx *ctx = owner->ctx;
    if (owner->deferred) return 0;
    nc_deferred *only = NULL;
    for (nc_deferred *d = ctx->deferred_head; d; d = d->next) {
        if (d->src[0] != owner && d->src[1] != owner && d->src[2] != owner) continue;
        if (only || d->kind != NC_DEF_UNARY || d->adopt || d->x != (const float *)owner->data) return 0;
        only = d;
    }
    if (!only) return 0;
    only->adopt = owner->data, only->adopt_bytes = owner->bytes;
    only->src[0] = NULL;
    return 1;
}

void nc__materialize(nc_tensor *owner) {
    nc_deferred *d = owner->deferred;
    if (!d) return;
    nc_ctx *ctx = owner->ctx;
    unlink_deferred(ctx, d); /* first: the launch below reads no recipe */
    if (d->kind == NC_DEF_ATTN) nck_attn_probs(nc__k(ctx), &d->at, (float *)owner->data);
    else if (d->kind == NC_DEF_UNARY) {
        nck_unary_fwd(nc__k(ctx), d->act, d->act_s, d->x, (float *)owner->data, d->N);
        free_adopted(ctx, d);
    }
    else
        nck_bn_apply(nc__k(ctx), d->x, d->w, d->b, d->mean, d->invstd, (float *)owner->data, d->N, d->C, d->S,
                     d->act, d->act_s);
}

void nc__deferred_release(nc_tensor *owner) {
    nc_ctx *ctx = owner->ctx;
    if (!ctx->deferred_head) return;
    for (nc_deferred *d = ctx->deferred_head, *next; d; d = next) {
        next = d->next;
        if ((d->src[0] == owner || d->src[1] == owner || d->src[2] == owner) && d->owner != owner)
            nc__materialize(d->owner);
    }
    if (owner->deferred) {
        nc_deferred *d = owner->deferred;
        unlink_deferred(ctx, d);
        free_adopted(ctx, d);
    }
}

void nc__deferred_flush(nc_ctx *ctx) {
    while (ctx->deferred_head) nc__materialize(ctx->deferred_head->owner);
}

void nc__deferred_reset(nc_ctx *ctx) {
    for (nc_deferred *d = ctx->deferred_head; d; d = d->next) d->owner->deferred = NULL;
    ctx->deferred_head = NULL;
}

/* ---- activations consumed on the fly --------------------------------------------------------- */

int nc__defer_unary(nc_tensor *out, nc_tensor *x, int act, float act_s) {
    nc_ctx *ctx = out->ctx;
    if (!ctx->fuse || ctx->fwd_on_tape || nc__deferred_of(x) || !nc_is_contiguous(x) || x->dtype != NC_F32) return 0;
    nc_deferred *d = (nc_deferred *)nc__meta_alloc(ctx, sizeof(nc_deferred), 0);
    if (!d) return 0;
    memset(d, 0, sizeof *d);
    d->owner = out, d->src[0] = nc__owner(x), d->kind = NC_DEF_UNARY;
    d->x = (const float *)nc__dev(x), d->act = act, d->act_s = act_s, d->N = nc_numel(x);
    d->next = ctx->deferred_head;
    ctx->deferred_head = d;
    out->deferred = d;
    return 1;
}

int nc__unary_recipe(const nc_tensor *t, const float **x, int *act, float *act_s) {
    const nc_deferred *d = nc__deferred_of(t);
    if (!d || d->kind != NC_DEF_UNARY) return 0;
    *x = d->x, *act = d->act, *act_s = d->act_s;
    return 1;
}

/* ---- attention chains --------------------------------------------------------------------------- */
/* newch's multi-head attention runs scores = q @ k^T, masked_fill, softmax, dropout and probs @ v as
 * separate ops (newch/net/__init__.py:811-820). Here the scores and each following tensor of the chain
 * are recipes (nck_attn at the chain's stage); the product with v runs the fused kernel, which forms
 * the probabilities on chip. A reader of any chain tensor materialises it (nck_attn_probs). */

/* t's leading dims folded into one batch dim: element (b, r, c) at data + b s[0] + r s[1] + c s[2] */
static int view3(const nc_tensor *t, int64_t *B, int64_t s[3]) {
    const int nd = t->ndim;
    if (nd < 3 || t->dtype != NC_F32) return 0;
    int64_t b = 1, bs = 0;
    for (int i = nd - 3; i >= 0; i--) {
        if (t->shape[i] == 1) continue;
        if (b == 1) bs = t->stride[i];
        else if (t->stride[i] != bs * b) return 0;
        b *= t->shape[i];
    }
    *B = b, s[0] = bs, s[1] = t->stride[nd - 2], s[2] = t->stride[nd - 1];
    return 1;
}

static int same_batch(const nc_tensor *a, const nc_tensor *b) {
    if (a->ndim != b->ndim) return 0;
    for (int i = 0; i < a->ndim - 2; i++)
        if (a->shape[i] != b->shape[i]) return 0;
    return 1;
}

static const nc_deferred *attn_of(const nc_tensor *t) {
    const nc_deferred *r = nc__deferred_of(t);
    return r && r->kind == NC_DEF_ATTN ? r : NULL;
}

static nc_deferred *attn_new(nc_ctx *ctx, nc_tensor *out, const nc_deferred *from) {
    nc_deferred *d = (nc_deferred *)nc__meta_alloc(ctx, sizeof(nc_deferred), 0);
    if (!d) return NULL;
    if (from) *d = *from;
    else memset(d, 0, sizeof *d);
    d->owner = out, d->kind = NC_DEF_ATTN;
    d->next = ctx->deferred_head;
    ctx->deferred_head = d;
    out->deferred = d;
    return d;
}

int nc__attn_bmm(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    nc_ctx *ctx = o->ctx;
    if (!ctx->fuse || !nc_is_contiguous(o)) return 0;
    const int nd = a->ndim;
    int64_t Ba, Bb, sa[3], sb[3];
    const nc_deferred *r = attn_of(a);
    if (r) { /* probabilities @ v */
        if (r->at.stage < NCK_ATT_SOFTMAX || !same_batch(a, b) || !view3(b, &Bb, sb) || Bb != r->at.B ||
            b->shape[nd - 2] != r->at.S || !nck_attn_ok(r->at.L, r->at.S, r->at.D, b->shape[nd - 1]))
            return 0;
        nck_attn at = r->at;
        at.v = (const float *)nc__dev(b);
        memcpy(at.vs, sb, sizeof sb);
        at.Dv = b->shape[nd - 1];
        nck_attn_fwd(nc__k(ctx), &at, (float *)o->data);
        return 1;
    }
    /* scores: a [.., L, D] @ b [.., D, S], the same batch dims */
    if (nc__deferred_of(a) || nc__deferred_of(b) || !same_batch(a, b) || !view3(a, &Ba, sa) || !view3(b, &Bb, sb))
        return 0;
    const int64_t L = a->shape[nd - 2], D = a->shape[nd - 1], S = b->shape[nd - 1];
    if (!nck_attn_ok(L, S, D, 1) || Ba < 1) return 0;
    nc_deferred *d = attn_new(ctx, o, NULL);
    if (!d) return 0;
    d->src[0] = nc__owner(a), d->src[1] = nc__owner(b);
    nck_attn *at = &d->at;
    at->q = (const float *)nc__dev(a);
    at->k = (const float *)nc__dev(b);
    memcpy(at->qs, sa, sizeof sa);
    at->ks[0] = sb[0], at->ks[1] = sb[2], at->ks[2] = sb[1]; /* K (b, j, d) = b (b, d, j) */
    at->B = Ba, at->L = L, at->S = S, at->D = D, at->Dv = 0;
    at->stage = NCK_ATT_SCORES, at->scale = 1.0f;
    return 1;
}

int nc__attn_scale(nc_node *n, float s) {
    const nc_deferred *r = attn_of(n->in[0]);
    if (!r || r->at.stage != NCK_ATT_SCORES || r->at.scaled) return 0;
    nc_deferred *d = attn_new(n->out->ctx, n->out, r);
    if (!d) return 0;
    d->at.scaled = 1, d->at.scale = s;
    return 1;
}

/* the mask's strides over the chain's (b, i, j) when it broadcasts there by strides alone */
static int mask_strides(const nc_tensor *m, const nc_tensor *x, const nck_attn *at, int64_t ms[3]) {
    const int nm = m->ndim, nx = x->ndim;
    if (m->dtype != NC_I32 || nm > nx) return 0;
    for (int k = 0; k < 2; k++) { /* the last two dims */
        const int im = nm - 1 - k;
        const int64_t ext = k == 0 ? at->S : at->L;
        int64_t *dst = &ms[2 - k];
        if (im < 0 || m->shape[im] == 1) *dst = 0;
        else if (m->shape[im] == ext) *dst = m->stride[im];
        else return 0;
    }
    /* batch dims: all broadcast, or exactly x's */
    int all_one = 1;
    for (int i = 0; i < nm - 2; i++) all_one &= m->shape[i] == 1;
    if (all_one) {
        ms[0] = 0;
        return 1;
    }
    if (nm != nx) return 0;
    for (int i = 0; i < nm - 2; i++)
        if (m->shape[i] != x->shape[i]) return 0;
    /* fold m's batch dims as view3 does */
    int64_t b = 1, bs = 0;
    for (int i = nm - 3; i >= 0; i--) {
        if (m->shape[i] == 1) continue;
        if (b == 1) bs = m->stride[i];
        else if (m->stride[i] != bs * b) return 0;
        b *= m->shape[i];
    }
    if (b != at->B) return 0;
    ms[0] = bs;
    return 1;
}

int nc__attn_mask(nc_node *n) {
    nc_tensor *x = n->in[0], *m = n->in[1];
    const nc_deferred *r = attn_of(x);
    int64_t ms[3];
    if (!r || r->at.stage != NCK_ATT_SCORES || !mask_strides(m, x, &r->at, ms)) return 0;
    nc_deferred *d = attn_new(n->out->ctx, n->out, r);
    if (!d) return 0;
    d->src[2] = nc__owner(m);
    d->at.mask = (const int32_t *)nc__dev(m);
    memcpy(d->at.ms, ms, sizeof ms);
    d->at.fill = n->p.f[0];
    d->at.stage = NCK_ATT_MASKED;
    return 1;
}

int nc__attn_softmax(nc_node *n) {
    const nc_deferred *r = attn_of(n->in[0]);
    if (!r || r->at.stage > NCK_ATT_MASKED) return 0;
    nc_deferred *d = attn_new(n->out->ctx, n->out, r);
    if (!d) return 0;
    d->at.stage = NCK_ATT_SOFTMAX;
    return 1;
}

int nc__attn_dropout(nc_node *n, const uint32_t *bits) {
    const nc_deferred *r = attn_of(n->in[0]);
    if (!r || r->at.stage != NCK_ATT_SOFTMAX) return 0;
    nc_deferred *d = attn_new(n->out->ctx, n->out, r);
    if (!d) return 0;
    d->at.bits = bits, d->at.p = n->p.f[0];
    d->at.stage = NCK_ATT_DROPOUT;
    return 1;
}

int nc__attn_dropout_ok(const nc_tensor *x) {
    const nc_deferred *r = attn_of(x);
    return r && r->at.stage == NCK_ATT_SOFTMAX;
}

/* ---- fused backward chains ---------------------------------------------------------------------- */

/* t is an intermediate whose only consumer in this pass is one node and whose values were never read */
static int private_recipe(const nc_tensor *t, uint32_t epoch) {
    return nc__deferred_of(t) && t->use_epoch == epoch && t->uses == 1 && t->node;
}

static int is_bn_training(const nc_node *n) { return n->op == &nc_op_batch_norm && n->p.i[0] == 1; }

static int is_bn_recipe(const nc_tensor *t) { return t->deferred->kind == NC_DEF_BN; }

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
    if (!private_recipe(z, ep) || !is_bn_recipe(z)) return 0;
    const nc_deferred *rz = z->deferred;
    nc_node *na = NULL, *nb = z->node;
    if (rz->act >= 0) {
        na = z->node;
        if (nc__unary_kind(na->op) != rz->act || na->fused == ep) return 0;
        nc_tensor *y = na->in[0];
        if (!private_recipe(y, ep) || !is_bn_recipe(y) || y->deferred->act >= 0) return 0;
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
    nck_bn_pool_bwd(nc__k(ctx), X, w, b, (const float *)np->out->grad->data, (const int32_t *)np->saved,
                    nc__pool_xarg(np), sv->mean, sv->invstd, gx, gw, gb, x->shape[0], x->shape[1], x->shape[2],
                    x->shape[3], acc, rz->act, rz->act_s);
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
    if (!private_recipe(y, ep) || !is_bn_recipe(y) || y->deferred->act >= 0) return 0;
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

/* probabilities @ v over an attention chain whose tensors nothing else read: one fused backward
 * gives dq, dk and dv; the chain's dropout, softmax, mask, scale and scores nodes are consumed */
static int fuse_attn_chain(nc_ctx *ctx, nc_node *n2, nc_node **consumed) {
    if (n2->op != &nc_op_bmm) return 0;
    const uint32_t ep = ctx->mark_epoch;
    nc_tensor *p = n2->in[0], *v = n2->in[1];
    if (!private_recipe(p, ep) || p->deferred->kind != NC_DEF_ATTN) return 0;
    const nc_deferred *r = p->deferred;
    int64_t Bv, vs[3];
    const int nd = v->ndim;
    if (r->at.stage < NCK_ATT_SOFTMAX || !view3(v, &Bv, vs) || Bv != r->at.B || v->shape[nd - 2] != r->at.S ||
        !nck_attn_ok(r->at.L, r->at.S, r->at.D, v->shape[nd - 1]))
        return 0;
    int k = 0;
    nc_tensor *t = p;
    nc_node *n1 = NULL;
    while (!n1) {
        nc_node *nt = t->node;
        if (!nt || nt->fused == ep || k >= NC_CHAIN_MAX - 1) return 0;
        if (nt->op == &nc_op_bmm) {
            n1 = nt;
            break;
        }
        consumed[k++] = nt;
        t = nt->in[0];
        if (!private_recipe(t, ep) || t->deferred->kind != NC_DEF_ATTN) return 0;
    }
    consumed[k++] = n1;
    nc_tensor *q = n1->in[0], *kt = n1->in[1];
    nck_attn at = r->at;
    at.v = (const float *)nc__dev(v);
    memcpy(at.vs, vs, sizeof vs);
    at.Dv = v->shape[nd - 1];
    float *dq = NULL, *dk = NULL, *dv = NULL;
    int aq = 0, ak = 0, av = 0;
    if (nc__needs_grad(q)) {
        nc_tensor *g = nc__grad_buf_acc(q, &aq);
        dq = g ? (float *)g->data : NULL;
    }
    if (nc__needs_grad(kt)) {
        nc_tensor *g = nc__grad_buf_acc(kt, &ak);
        dk = g ? (float *)g->data : NULL;
    }
    if (nc__needs_grad(v)) {
        nc_tensor *g = nc__grad_buf_acc(v, &av);
        dv = g ? (float *)g->data : NULL;
    }
    nck_attn_bwd(nc__k(ctx), &at, (const float *)n2->out->grad->data, dq, aq, dk, ak, dv, av);
    return k;
}

int nc__fused_backward(nc_ctx *ctx, nc_node *n, nc_node **consumed) {
    if (!ctx->fuse || !n->out->grad) return 0;
    int k = fuse_pool_chain(ctx, n, consumed);
    if (!k) k = fuse_act_chain(ctx, n, consumed);
    if (!k) k = fuse_attn_chain(ctx, n, consumed);
    return k;
}

void nc__backward_inputs(nc_node *n) {
    if (!n->out->ctx->deferred_head) return;
    if (nc__owner(n->out)->deferred) nc__materialize(nc__owner(n->out));
    for (int i = 0; i < n->n_in; i++)
        if (n->in[i] && nc__owner(n->in[i])->deferred) nc__materialize(nc__owner(n->in[i]));
}
