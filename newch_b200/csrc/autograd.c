/* Eager execution and tape autograd, with every node's work enqueued on the context's stream.
 *
 * Same contract as newch engine/src/autograd/autograd.c: nc__apply (:12-82) validates, infers,
 * allocates, runs forward and records a node when an input needs grad; nc_backward_ex (:107-183)
 * marks the nodes that reach the loss, zeroes intermediate grads, seeds d(loss) = 1 and runs the
 * marked nodes newest-first, handing each node's temporaries, its output grad and (with
 * FREE_GRAPH) its dead output back to the arena right after it. On the device this is a stream
 * schedule: the host walks the tape and enqueues kernels without waiting; arena blocks released
 * during the walk are re-used by later kernels of the same stream, so stream order keeps them safe.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>

nc_tensor *nc__apply(const nc_op_def *op, nc_tensor **in, int n_in, const nc_op_params *p) {
    for (int i = 0; i < n_in; i++)
        if (!in[i]) return NULL;
    nc_ctx *ctx = in[0]->ctx;
    if (ctx->status != NC_OK) return NULL;
    for (int i = 1; i < n_in; i++) {
        if (in[i]->ctx != ctx) {
            nc__error(ctx, NC_ERR_ARG, "%s: inputs belong to different contexts", op->name);
            return NULL;
        }
    }
    int persistent = nc__is_persistent_mode(ctx);
    nc_node *n = (nc_node *)nc__meta_alloc(ctx, sizeof(nc_node), 0);
    if (!n) return NULL;
    n->op = op;
    n->n_in = n_in;
    for (int i = 0; i < n_in; i++) n->in[i] = in[i];
    if (p) n->p = *p;

    nc_dtype dt;
    int nd = 0;
    int64_t shape[NC_MAX_DIMS];
    if (op->infer(n, &dt, &nd, shape) != NC_OK) return NULL;

    int record = ctx->grad_enabled && !persistent && op->backward != NULL;
    if (record) {
        record = 0;
        for (int i = 0; i < n_in; i++)
            if (nc__needs_grad(in[i])) record = 1;
    }
    int can_view = op->view != NULL && !persistent;
    if (!(can_view && op->view(n, nd, shape))) {
        for (int i = 0; i < n_in; i++) nc__dev(in[i]); /* host writes reach the device first */
        n->out = nc__tensor_new(ctx, dt, nd, shape, persistent);
        if (!n->out) return NULL;
        int scratch = !record && !persistent && !ctx->bwd_logging;
        if (scratch) {
            ctx->bwd_logging = 1;
            ctx->bwd_tmp_n = 0;
        }
        nc_status st = op->forward(n);
        if (scratch) {
            ctx->bwd_logging = 0;
            for (int i = 0; i < ctx->bwd_tmp_n; i++) nc__arena_free(ctx, ctx->bwd_tmp[i], ctx->bwd_tmp_size[i]);
            ctx->bwd_tmp_n = 0;
            n->saved = NULL;
        }
        if (st != NC_OK) return NULL;
    }
    if (!n->out) return NULL;
    if (record) {
        for (int i = 0; i < n_in; i++) nc__owner(in[i])->flags |= NC_TF_ON_TAPE;
        nc__owner(n->out)->flags |= NC_TF_ON_TAPE;
        n->out->flags |= NC_TF_REQUIRES_GRAD;
        n->out->node = n;
        n->prev = ctx->tape;
        ctx->tape = n;
    }
    return n->out;
}

static int cmp_ptr(const void *a, const void *b) {
    uintptr_t x = (uintptr_t) * (void *const *)a, y = (uintptr_t) * (void *const *)b;
    return x < y ? -1 : x > y;
}

static int is_kept(void *const *kept, int n, void *data) {
    return n > 0 && bsearch(&data, kept, (size_t)n, sizeof(void *), cmp_ptr) != NULL;
}

nc_status nc_backward(nc_tensor *loss) { return nc_backward_ex(loss, 0, NULL, 0); }

void nc_release_temp(nc_tensor *t) {
    if (!t || (t->flags & (NC_TF_PERSISTENT | NC_TF_ON_TAPE)) || !(t->flags & NC_TF_OWNS_DATA) || !t->data) return;
    nc_ctx *ctx = t->ctx;
    nc__arena_free(ctx, t->data, t->bytes);
    t->data = NULL;
    t->coh = 0;
    if (t->grad && t->grad->data && !(t->grad->flags & NC_TF_PERSISTENT)) {
        nc__arena_free(ctx, t->grad->data, t->grad->bytes);
        t->grad->data = NULL;
        t->grad = NULL;
    }
}

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
    uint32_t ep = ++ctx->mark_epoch;
    if (loss->node) loss->node->mark = ep;
    for (nc_node *n = ctx->tape; n; n = n->prev) {
        if (n->mark != ep) continue;
        if (n->released) {
            nc__error(ctx, NC_ERR_STATE,
                      "backward: part of this graph was released by an earlier backward "
                      "(use retain_graph=True on the first backward to run it twice)");
            return ctx->status;
        }
        for (int i = 0; i < n->n_in; i++)
            if (n->in[i]->node && nc__needs_grad(n->in[i])) n->in[i]->node->mark = ep;
    }
    int retain = (flags & NC_BACKWARD_RETAIN) != 0, free_graph = !retain && (flags & NC_BACKWARD_FREE_GRAPH);

    void **kept = NULL;
    int nk = 0;
    if (free_graph && n_keep > 0) {
        kept = (void **)malloc(sizeof(void *) * (size_t)n_keep);
        if (!kept) {
            nc__error(ctx, NC_ERR_OOM, "backward: out of memory");
            return ctx->status;
        }
        for (int i = 0; i < n_keep; i++)
            if (keep[i]) kept[nk++] = keep[i]->data;
        qsort(kept, (size_t)nk, sizeof(void *), cmp_ptr);
    }
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    for (nc_node *n = ctx->tape; n; n = n->prev)
        if (n->mark == ep && n->out->grad && n->out->grad->data) {
            cudaMemsetAsync(n->out->grad->data, 0, n->out->grad->bytes, s);
            n->out->grad->coh &= ~NC_COH_HOST_VALID;
        }

    int seed_acc;
    nc_tensor *g = nc__grad_buf_acc(loss, &seed_acc);
    if (!g) {
        free(kept);
        return ctx->status;
    }
    /* d loss / d loss = 1: stored into a fresh buffer, added to one that already holds a gradient */
    if (seed_acc) nck_add_scalar_inplace(nc__k(ctx), (float *)g->data, 1.0f);
    else nck_fill_f32(nc__k(ctx), (float *)g->data, 1.0f, nc_numel(loss));

    for (nc_node *n = ctx->tape; n; n = n->prev) {
        if (n->mark != ep || !n->out->grad) continue;
        ctx->bwd_logging = !retain;
        ctx->bwd_tmp_n = 0;
        n->op->backward(n);
        ctx->bwd_logging = 0;
        if (retain) continue;
        for (int i = 0; i < ctx->bwd_tmp_n; i++) nc__arena_free(ctx, ctx->bwd_tmp[i], ctx->bwd_tmp_size[i]);
        ctx->bwd_tmp_n = 0;
        nc_tensor *o = n->out, *og = o->grad;
        nc__arena_free(ctx, og->data, og->bytes);
        o->grad = NULL;
        if (free_graph && o != loss && (o->flags & NC_TF_OWNS_DATA) && !(o->flags & NC_TF_PERSISTENT) &&
            !is_kept(kept, nk, o->data)) {
            nc__arena_free(ctx, o->data, o->bytes);
            o->data = NULL;
            n->released = 1;
        }
    }
    free(kept);
    nc__cuda_ok(ctx, cudaGetLastError(), "backward");
    return ctx->status;
}

void nc_zero_grad(nc_tensor *t) {
    if (t && t->grad && !(t->flags & NC_TF_GRAD_CLEARED)) {
        nc__dev_write(t->grad);
        cudaMemsetAsync(t->grad->data, 0, t->grad->bytes, (cudaStream_t)t->ctx->dev.stream);
    }
}

void nc_clear_grad(nc_tensor *t) {
    if (t && t->grad) t->flags |= NC_TF_GRAD_CLEARED;
}
