/* Eager op execution and reverse-mode autograd for the B200 engine.
 *
 * Contract (newch engine/src/autograd/autograd.c): nc__apply (:12-82) is the single entry of every
 * op and fails in infer before anything is launched; nc_backward_ex (:107-183) accumulates
 * d(loss)/d(input) into every tensor that reaches the loss, releasing each node's temporaries, its
 * output gradient and (FREE_GRAPH, unless kept) its dead output as soon as the node is done; errors
 * and messages are newch's, because its Python layer reads them.
 *
 * How it runs here. Forward ops enqueue kernels on the context's stream and return at once. A
 * backward pass is compiled into a schedule before anything is enqueued:
 *   1. the live set: a depth-first search from the loss over inputs that need a gradient (work in
 *      proportion to the graph that reaches the loss, not to everything recorded in the step);
 *   2. the order: live nodes by descending recording sequence, a topological order of the reversed
 *      graph, so each node runs after every consumer of its output;
 *   3. leaf accounting: for every leaf (a tensor with no producing node) the number of live nodes
 *      that write its gradient. The schedule walk reports a leaf final once its last writer is
 *      enqueued, which lets data-parallel runs start all-reducing finished gradient buckets on a
 *      communication stream while the remaining nodes still run (optim.c, dp.c).
 * The walk then enqueues each node's backward kernels on the stream without waiting. Arena blocks
 * handed back during the walk are re-used by later kernels of the same stream, which stream order
 * makes safe.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>

/* ---- forward ---------------------------------------------------------------------------------- */

/* Allocations an op makes while running outside the tape (no node keeps its saved state) are
 * scratch: they go back to the arena when the op returns. Nested scopes are not opened (a forward
 * run from inside a backward already logs into the node's temporaries). */
typedef struct {
    int open;
} scratch_scope;

static void scratch_open(nc_ctx *ctx, scratch_scope *sc, int wanted) {
    sc->open = wanted && !ctx->bwd_logging;
    if (sc->open) {
        ctx->bwd_logging = 1;
        ctx->bwd_tmp_n = 0;
    }
}

static void scratch_close(nc_ctx *ctx, scratch_scope *sc, nc_node *n) {
    if (!sc->open) return;
    ctx->bwd_logging = 0;
    for (int i = 0; i < ctx->bwd_tmp_n; i++) nc__arena_free(ctx, ctx->bwd_tmp[i], ctx->bwd_tmp_size[i]);
    ctx->bwd_tmp_n = 0;
    n->saved = NULL;
}

/* the context of a call whose inputs are all present and agree, else NULL (sticky errors included) */
static nc_ctx *inputs_context(const nc_op_def *op, nc_tensor **in, int n_in) {
    for (int i = 0; i < n_in; i++)
        if (!in[i]) return NULL; /* a failed producer: pass the NULL on */
    nc_ctx *ctx = in[0]->ctx;
    if (ctx->status != NC_OK) return NULL;
    for (int i = 1; i < n_in; i++)
        if (in[i]->ctx != ctx) {
            nc__error(ctx, NC_ERR_ARG, "%s: inputs belong to different contexts", op->name);
            return NULL;
        }
    return ctx;
}

static int wants_node(const nc_ctx *ctx, const nc_op_def *op, nc_tensor **in, int n_in, int persistent) {
    if (!ctx->grad_enabled || persistent || !op->backward) return 0;
    for (int i = 0; i < n_in; i++)
        if (nc__needs_grad(in[i])) return 1;
    return 0;
}

static void record_node(nc_ctx *ctx, nc_node *n) {
    for (int i = 0; i < n->n_in; i++) nc__owner(n->in[i])->flags |= NC_TF_ON_TAPE;
    nc__owner(n->out)->flags |= NC_TF_ON_TAPE;
    n->out->flags |= NC_TF_REQUIRES_GRAD;
    n->out->node = n;
    n->seq = ++ctx->node_seq;
    n->prev = ctx->tape;
    ctx->tape = n;
}

nc_tensor *nc__apply(const nc_op_def *op, nc_tensor **in, int n_in, const nc_op_params *p) {
    nc_ctx *ctx = inputs_context(op, in, n_in);
    if (!ctx) return NULL;
    const int persistent = nc__is_persistent_mode(ctx);
    nc_node *n = (nc_node *)nc__meta_alloc(ctx, sizeof(nc_node), 0);
    if (!n) return NULL;
    n->op = op;
    n->n_in = n_in;
    memcpy(n->in, in, sizeof(nc_tensor *) * (size_t)n_in);
    if (p) n->p = *p;

    nc_dtype dt;
    int nd = 0;
    int64_t shape[NC_MAX_DIMS];
    if (op->infer(n, &dt, &nd, shape) != NC_OK) return NULL; /* nothing launched yet */

    const int on_tape = wants_node(ctx, op, in, n_in, persistent);
    const int viewed = op->view && !persistent && op->view(n, nd, shape);
    if (!viewed) {
        for (int i = 0; i < n_in; i++) /* host-side writes reach the device first */
            if (!(op->flags & NC_OPF_RECIPE) || !nc__deferred_of(in[i])) nc__dev(in[i]);
        n->out = nc__tensor_new(ctx, dt, nd, shape, persistent);
        if (!n->out) return NULL;
        scratch_scope sc;
        scratch_open(ctx, &sc, !on_tape && !persistent);
        const int was = ctx->fwd_on_tape;
        ctx->fwd_on_tape = on_tape;
        nc_status st = op->forward(n);
        ctx->fwd_on_tape = was;
        scratch_close(ctx, &sc, n);
        if (st != NC_OK) return NULL;
    }
    if (!n->out) return NULL;
    if (on_tape) record_node(ctx, n);
    return n->out;
}

/* ---- small host containers -------------------------------------------------------------------- */

typedef struct {
    nc_node **v;
    int n, cap;
} node_vec;

static int node_push(node_vec *a, nc_node *x) {
    if (a->n == a->cap) {
        int cap = a->cap ? 2 * a->cap : 64;
        nc_node **v = (nc_node **)realloc(a->v, sizeof(nc_node *) * (size_t)cap);
        if (!v) return 0;
        a->v = v;
        a->cap = cap;
    }
    a->v[a->n++] = x;
    return 1;
}

/* open-addressing set of data pointers (the tensors Python still holds) */
typedef struct {
    void **slot;
    size_t mask;
} ptr_set;

static size_t ptr_hash(const void *p) {
    uint64_t x = (uint64_t)(uintptr_t)p;
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 29;
    return (size_t)x;
}

static int ptr_set_build(ptr_set *s, nc_tensor *const *items, int n) {
    size_t cap = 16;
    while (cap < (size_t)n * 2) cap <<= 1;
    s->slot = (void **)calloc(cap, sizeof(void *));
    s->mask = cap - 1;
    if (!s->slot) return 0;
    for (int i = 0; i < n; i++) {
        void *d = items[i] ? items[i]->data : NULL;
        if (!d) continue;
        size_t h = ptr_hash(d) & s->mask;
        while (s->slot[h] && s->slot[h] != d) h = (h + 1) & s->mask;
        s->slot[h] = d;
    }
    return 1;
}

static int ptr_set_has(const ptr_set *s, const void *d) {
    if (!s->slot || !d) return 0;
    size_t h = ptr_hash(d) & s->mask;
    while (s->slot[h]) {
        if (s->slot[h] == d) return 1;
        h = (h + 1) & s->mask;
    }
    return 0;
}

/* ---- backward plan ---------------------------------------------------------------------------- */

typedef struct {
    node_vec order; /* live nodes, newest first */
    ptr_set keep;   /* data of tensors the caller still holds (FREE_GRAPH spares them) */
    uint32_t epoch;
} bw_plan;

static void plan_free(bw_plan *pl) {
    free(pl->order.v);
    free(pl->keep.slot);
}

static int by_seq_desc(const void *a, const void *b) {
    uint64_t x = (*(nc_node *const *)a)->seq, y = (*(nc_node *const *)b)->seq;
    return x < y ? 1 : x > y ? -1 : 0;
}

static int is_grad_leaf(const nc_tensor *t) { return !t->node && nc__needs_grad(t); }

/* Live set by depth-first search from the loss's node; leaves get their writer counts. Returns 0
 * (with the context error set) when the graph cannot be differentiated again or memory runs out. */
static int plan_collect(nc_ctx *ctx, nc_tensor *loss, bw_plan *pl) {
    const uint32_t ep = pl->epoch;
    node_vec stack = {0};
    int ok = 1;
    if (loss->node) {
        loss->node->mark = ep;
        ok = node_push(&stack, loss->node);
    }
    while (ok && stack.n) {
        nc_node *n = stack.v[--stack.n];
        if (n->released) {
            nc__error(ctx, NC_ERR_STATE,
                      "backward: part of this graph was released by an earlier backward "
                      "(use retain_graph=True on the first backward to run it twice)");
            ok = 0;
            break;
        }
        if (!node_push(&pl->order, n)) {
            ok = 0;
            break;
        }
        for (int i = 0; i < n->n_in; i++) {
            nc_tensor *x = n->in[i];
            if (x->use_epoch != ep) x->use_epoch = ep, x->uses = 0;
            x->uses++; /* consumers of x in this pass (a fused chain needs x to have one) */
            if (!nc__needs_grad(x)) continue;
            if (x->node) {
                if (x->node->mark != ep) {
                    x->node->mark = ep;
                    if (!node_push(&stack, x->node)) ok = 0;
                }
            } else {
                if (x->bw_epoch != ep) {
                    x->bw_epoch = ep;
                    x->bw_pending = 0;
                    nc__grad_expect(x);
                }
                x->bw_pending++;
            }
        }
    }
    free(stack.v);
    if (!ok && ctx->status == NC_OK) nc__error(ctx, NC_ERR_OOM, "backward: out of memory");
    if (ok && pl->order.n > 1) qsort(pl->order.v, (size_t)pl->order.n, sizeof(nc_node *), by_seq_desc);
    return ok;
}

/* A node's backward is enqueued: its leaf inputs lose one pending writer each. */
static void plan_node_done(nc_node *n) {
    for (int i = 0; i < n->n_in; i++) {
        nc_tensor *x = n->in[i];
        if (is_grad_leaf(x) && --x->bw_pending == 0) nc__grad_final(x);
    }
}

/* The node's own temporaries, its output gradient and (if nothing needs it) its output. */
static void plan_release_node(nc_ctx *ctx, nc_node *n, nc_tensor *loss, const bw_plan *pl, int free_graph) {
    for (int i = 0; i < ctx->bwd_tmp_n; i++) nc__arena_free(ctx, ctx->bwd_tmp[i], ctx->bwd_tmp_size[i]);
    ctx->bwd_tmp_n = 0;
    nc_tensor *o = n->out;
    if (o->grad) { /* a node run inside a fused chain never formed its output gradient */
        nc__arena_free(ctx, o->grad->data, o->grad->bytes);
        o->grad = NULL;
    }
    if (!free_graph || o == loss || !(o->flags & NC_TF_OWNS_DATA) || (o->flags & NC_TF_PERSISTENT)) return;
    if (ptr_set_has(&pl->keep, o->data)) return;
    nc__deferred_release(o); /* recipes reading o are computed first; o's own is dropped */
    nc__arena_free(ctx, o->data, o->bytes);
    o->data = NULL;
    n->released = 1;
}

nc_status nc_backward(nc_tensor *loss) { return nc_backward_ex(loss, 0, NULL, 0); }

nc_status nc_backward_ex(nc_tensor *loss, int flags, nc_tensor *const *keep, int n_keep) {
    if (!loss) return NC_ERR_ARG;
    nc_ctx *ctx = loss->ctx;
    if (ctx->status != NC_OK) return ctx->status;
    if (nc_numel(loss) != 1 || loss->dtype != NC_F32) {
        nc__error(ctx, NC_ERR_SHAPE, "backward: loss must be a single f32 element");
        return ctx->status;
    }
    if (!nc__needs_grad(loss)) {
        nc__error(ctx, NC_ERR_STATE,
                  "backward: loss does not require grad (no parameter reached it, or grad was disabled)");
        return ctx->status;
    }
    const int retain = (flags & NC_BACKWARD_RETAIN) != 0;
    const int free_graph = !retain && (flags & NC_BACKWARD_FREE_GRAPH) != 0;

    bw_plan pl;
    memset(&pl, 0, sizeof pl);
    pl.epoch = ++ctx->mark_epoch;
    nc__grad_pass_begin(ctx);
    if (!plan_collect(ctx, loss, &pl) ||
        (free_graph && n_keep > 0 && !ptr_set_build(&pl.keep, keep, n_keep))) {
        if (ctx->status == NC_OK) nc__error(ctx, NC_ERR_OOM, "backward: out of memory");
        plan_free(&pl);
        return ctx->status;
    }

    /* gradients of intermediate tensors start from zero in every pass */
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    for (int k = 0; k < pl.order.n; k++) {
        nc_tensor *g = pl.order.v[k]->out->grad;
        if (g && g->data) {
            cudaMemsetAsync(g->data, 0, g->bytes, s);
            g->coh &= ~NC_COH_HOST_VALID;
        }
    }

    /* d loss / d loss = 1: stored into a fresh buffer, added to one that already holds a gradient */
    int seed_acc;
    nc_tensor *g = nc__grad_buf_acc(loss, &seed_acc);
    if (!g) {
        plan_free(&pl);
        return ctx->status;
    }
    if (seed_acc) nck_add_scalar_inplace(nc__k(ctx), (float *)g->data, 1.0f);
    else nck_fill_f32(nc__k(ctx), (float *)g->data, 1.0f, nc_numel(loss));
    if (is_grad_leaf(loss) && loss->bw_epoch != pl.epoch) {
        /* a leaf loss: its own gradient is the seed */
        loss->bw_epoch = pl.epoch;
        loss->bw_pending = 0;
        nc__grad_expect(loss);
        nc__grad_final(loss);
    }

    for (int k = 0; k < pl.order.n; k++) {
        nc_node *n = pl.order.v[k];
        if (n->fused == pl.epoch) { /* its backward ran inside a fused chain */
            if (!retain) plan_release_node(ctx, n, loss, &pl, free_graph);
            plan_node_done(n);
            continue;
        }
        if (n->out->grad) { /* else nothing flowed into this node */
            ctx->bwd_logging = !retain;
            ctx->bwd_tmp_n = 0;
            nc_node *chain[NC_CHAIN_MAX];
            const int nc = nc__fused_backward(ctx, n, chain);
            for (int c = 0; c < nc; c++) chain[c]->fused = pl.epoch;
            if (!nc) {
                nc__backward_inputs(n); /* an unfused backward reads real values */
                n->op->backward(n);
            }
            ctx->bwd_logging = 0;
            if (!retain) plan_release_node(ctx, n, loss, &pl, free_graph);
        }
        plan_node_done(n);
    }
    plan_free(&pl);
    nc__cuda_ok(ctx, cudaGetLastError(), "backward");
    return ctx->status;
}

/* ---- gradient resets -------------------------------------------------------------------------- */

void nc_zero_grad(nc_tensor *t) {
    if (!t || !t->grad || (t->flags & NC_TF_GRAD_CLEARED)) return;
    nc__dev_write(t->grad);
    cudaMemsetAsync(t->grad->data, 0, t->grad->bytes, (cudaStream_t)t->ctx->dev.stream);
}

void nc_clear_grad(nc_tensor *t) {
    if (t && t->grad) t->flags |= NC_TF_GRAD_CLEARED;
}

/* A temporary the caller no longer needs: its data (and gradient) go back to the arena now, unless
 * a recorded node still refers to it. */
void nc_release_temp(nc_tensor *t) {
    if (!t || (t->flags & (NC_TF_PERSISTENT | NC_TF_ON_TAPE)) || !(t->flags & NC_TF_OWNS_DATA) || !t->data) return;
    nc_ctx *ctx = t->ctx;
    if (!nc__deferred_adopt(t)) { /* else a pending recipe still reads the block and frees it later */
        nc__deferred_release(t);
        nc__arena_free(ctx, t->data, t->bytes);
    }
    t->data = NULL;
    t->coh = 0;
    nc_tensor *g = t->grad;
    if (g && g->data && !(g->flags & NC_TF_PERSISTENT)) {
        nc__arena_free(ctx, g->data, g->bytes);
        g->data = NULL;
        t->grad = NULL;
    }
}
