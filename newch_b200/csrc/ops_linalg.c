/* Dense contractions: matmul (leading dims of a folded into M), batched matmul with broadcast batch
 * dims, and the fused linear layer y = x W^T + b.
 *
 * Operand handling follows newch engine/src/ops/ops_linalg.c: transposed views go to the GEMM as
 * transpose flags instead of copies (as_gemm :17-30, bmm operands :138-160), gradients are the same
 * GEMMs (matmul :69-92, bmm :236-267, linear :311-331). The batched forms run as one strided-batch
 * GEMM launch whenever the batch dims collapse to one stride per operand; a broadcast operand's
 * gradient sums over the broadcast batch inside the GEMM (reduce_batch), without atomics.
 */
#include "nc_internal.h"

#include <stdio.h>

typedef struct {
    const float *p;
    int trans;
    int64_t ld;
} gemm_operand;

static gemm_operand as_gemm(nc_tensor *t, int64_t rows, int64_t cols) {
    gemm_operand g;
    if (t->ndim == 2 && t->stride[1] == 1 && t->stride[0] >= cols) {
        g.p = (const float *)nc__dev(t), g.trans = 0, g.ld = t->stride[0];
    } else if (t->ndim == 2 && t->stride[0] == 1 && t->stride[1] >= rows) {
        g.p = (const float *)nc__dev(t), g.trans = 1, g.ld = t->stride[1];
    } else {
        g.p = nc__contig_f32(t), g.trans = 0, g.ld = cols;
    }
    return g;
}

void nc__gemm(nc_ctx *ctx, int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
              const float *B, int64_t ldb, float beta, float *C, int64_t ldc) {
    nck_gemm_args a;
    memset(&a, 0, sizeof a);
    a.ta = ta, a.tb = tb, a.M = M, a.N = N, a.K = K, a.alpha = alpha, a.beta = beta;
    a.A = A, a.lda = lda, a.B = B, a.ldb = ldb, a.C = C, a.ldc = ldc;
    a.batch = 1;
    nck_gemm(nc__k(ctx), &a);
}

void nc__gemm_batched(nc_ctx *ctx, const nck_gemm_args *a) { nck_gemm(nc__k(ctx), a); }

/* ---- matmul: a [..., M, K] @ b [K, N] ------------------------------------------------------------ */

static nc_status matmul_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    if (!nc__expect_f32(n, 0) || !nc__expect_f32(n, 1)) return NC_ERR_DTYPE;
    if (a->ndim < 2 || b->ndim != 2 || a->shape[a->ndim - 1] != b->shape[0]) {
        char sa[96], sb[96];
        nc__error(a->ctx, NC_ERR_SHAPE, "matmul: cannot multiply %s by %s (expected [..., M, K] @ [K, N])",
                  nc__shape_str(a->ndim, a->shape, sa, sizeof sa), nc__shape_str(b->ndim, b->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = a->ndim;
    memcpy(shape, a->shape, sizeof(int64_t) * (size_t)a->ndim);
    shape[a->ndim - 1] = b->shape[1];
    return NC_OK;
}

static void mm_dims(const nc_node *n, int64_t *M, int64_t *K, int64_t *N) {
    const nc_tensor *a = n->in[0], *b = n->in[1];
    *K = b->shape[0];
    *N = b->shape[1];
    *M = nc_numel(a) / (*K ? *K : 1);
}

static gemm_operand a_operand(nc_tensor *a, int64_t M, int64_t K) {
    if (a->ndim == 2) return as_gemm(a, M, K);
    gemm_operand g = {nc__contig_f32(a), 0, K};
    return g;
}

static nc_status matmul_fwd(nc_node *n) {
    int64_t M, K, N;
    mm_dims(n, &M, &K, &N);
    gemm_operand A = a_operand(n->in[0], M, K), B = as_gemm(n->in[1], K, N);
    if (!A.p || !B.p) return NC_ERR_OOM;
    nc__gemm(n->out->ctx, A.trans, B.trans, M, N, K, 1.0f, A.p, A.ld, B.p, B.ld, 0.0f, (float *)n->out->data, N);
    return NC_OK;
}

static void matmul_bwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    int64_t M, K, N;
    mm_dims(n, &M, &K, &N);
    const float *g = (const float *)n->out->grad->data;
    if (nc__needs_grad(a)) {
        gemm_operand B = as_gemm(b, K, N);
        int acc;
        nc_tensor *ga = B.p ? nc__grad_buf_acc(a, &acc) : NULL;
        if (ga && B.p)
            nc__gemm(a->ctx, 0, !B.trans, M, K, N, 1.0f, g, N, B.p, B.ld, acc ? 1.0f : 0.0f, (float *)ga->data, K);
    }
    if (nc__needs_grad(b)) {
        gemm_operand A = a_operand(a, M, K);
        int acc;
        nc_tensor *gb = A.p ? nc__grad_buf_acc(b, &acc) : NULL;
        if (gb && A.p)
            nc__gemm(a->ctx, !A.trans, 0, K, N, M, 1.0f, A.p, A.ld, g, N, acc ? 1.0f : 0.0f, (float *)gb->data, N);
    }
}

const nc_op_def nc_op_matmul = {"matmul", 0, 0, matmul_infer, NULL, matmul_fwd, matmul_bwd};

/* ---- batched matmul ------------------------------------------------------------------------------ */

typedef struct {
    int nb;
    int64_t shape[NC_MAX_DIMS];
    int64_t count;
} batch_dims;

static int batch_shape(const nc_tensor *a, const nc_tensor *b, batch_dims *bd) {
    int na = a->ndim - 2, nb = b->ndim - 2;
    bd->nb = na > nb ? na : nb;
    bd->count = 1;
    for (int i = 0; i < bd->nb; i++) {
        int ia = i - (bd->nb - na), ib = i - (bd->nb - nb);
        int64_t da = ia < 0 ? 1 : a->shape[ia], db = ib < 0 ? 1 : b->shape[ib];
        if (da != db && da != 1 && db != 1) return 0;
        bd->shape[i] = da == 1 ? db : da;
        bd->count *= bd->shape[i];
    }
    return 1;
}

static void batch_strides(const nc_tensor *t, const int64_t *st, const batch_dims *bd, int64_t *out) {
    int tb = t->ndim - 2;
    for (int i = 0; i < bd->nb; i++) {
        int j = i - (bd->nb - tb);
        out[i] = (j < 0 || t->shape[j] == 1) ? 0 : st[j];
    }
}

typedef struct {
    const float *p;
    int trans;
    int64_t ld;
    int64_t bst[NC_MAX_DIMS];
} bmm_operand;

static int bmm_operand_of(nc_tensor *t, const batch_dims *bd, bmm_operand *o) {
    int nd = t->ndim;
    int64_t rows = t->shape[nd - 2], cols = t->shape[nd - 1];
    const int64_t *st = t->stride;
    int64_t cs[NC_MAX_DIMS];
    if (t->stride[nd - 1] == 1 && t->stride[nd - 2] >= cols) {
        o->p = (const float *)nc__dev(t), o->trans = 0, o->ld = t->stride[nd - 2];
    } else if (t->stride[nd - 2] == 1 && t->stride[nd - 1] >= rows) {
        o->p = (const float *)nc__dev(t), o->trans = 1, o->ld = t->stride[nd - 1];
    } else {
        o->p = nc__contig_f32(t), o->trans = 0, o->ld = cols;
        if (!o->p) return 0;
        nc__contig_strides(nd, t->shape, cs);
        st = cs;
    }
    batch_strides(t, st, bd, o->bst);
    return 1;
}

static nc_status bmm_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    batch_dims bd;
    if (!nc__expect_f32(n, 0) || !nc__expect_f32(n, 1)) return NC_ERR_DTYPE;
    if (a->ndim < 2 || b->ndim < 2 || a->shape[a->ndim - 1] != b->shape[b->ndim - 2] || !batch_shape(a, b, &bd)) {
        char sa[96], sb[96];
        nc__error(a->ctx, NC_ERR_SHAPE, "matmul: cannot multiply %s by %s (expected [..., M, K] @ [..., K, N])",
                  nc__shape_str(a->ndim, a->shape, sa, sizeof sa), nc__shape_str(b->ndim, b->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = bd.nb + 2;
    memcpy(shape, bd.shape, sizeof(int64_t) * (size_t)bd.nb);
    shape[bd.nb] = a->shape[a->ndim - 2];
    shape[bd.nb + 1] = b->shape[b->ndim - 1];
    return NC_OK;
}

/* C_i (+)= op(A_i) op(B_i) over the batch. Batch dims are merged where every operand's strides
 * allow; the remaining outer dims (rare) become separate launches. When C has stride 0 on the
 * innermost remaining dim, that dim is summed inside one launch (reduce_batch). */
static void bmm_run(nc_ctx *ctx, const batch_dims *bd, int ta, int tb, int64_t M, int64_t N, int64_t K,
                    const float *A, int64_t lda, const int64_t *sa, const float *B, int64_t ldb, const int64_t *sb,
                    float *C, int64_t ldc, const int64_t *sc, float beta) {
    int nb = bd->nb;
    int64_t shp[NC_MAX_DIMS], xa[NC_MAX_DIMS], xb[NC_MAX_DIMS], xc[NC_MAX_DIMS];
    int m = 0;
    for (int i = 0; i < nb; i++) {
        if (bd->shape[i] == 1) continue;
        if (m > 0 && xa[m - 1] == sa[i] * bd->shape[i] && xb[m - 1] == sb[i] * bd->shape[i] &&
            xc[m - 1] == sc[i] * bd->shape[i]) {
            shp[m - 1] *= bd->shape[i];
            xa[m - 1] = sa[i], xb[m - 1] = sb[i], xc[m - 1] = sc[i];
            continue;
        }
        shp[m] = bd->shape[i], xa[m] = sa[i], xb[m] = sb[i], xc[m] = sc[i];
        m++;
    }
    nck_gemm_args a;
    memset(&a, 0, sizeof a);
    a.ta = ta, a.tb = tb, a.M = M, a.N = N, a.K = K, a.alpha = 1.0f, a.beta = beta;
    a.lda = lda, a.ldb = ldb, a.ldc = ldc;
    if (m == 0) {
        a.A = A, a.B = B, a.C = C, a.batch = 1;
        nck_gemm(nc__k(ctx), &a);
        return;
    }
    int64_t outer = 1;
    for (int i = 0; i < m - 1; i++) outer *= shp[i];
    a.batch = shp[m - 1];
    a.sA = xa[m - 1], a.sB = xb[m - 1], a.sC = xc[m - 1];
    a.reduce_batch = xc[m - 1] == 0;
    for (int64_t o = 0; o < outer; o++) {
        int64_t rem = o, offa = 0, offb = 0, offc = 0;
        for (int i = m - 2; i >= 0; i--) {
            int64_t idx = rem % shp[i];
            rem /= shp[i];
            offa += idx * xa[i], offb += idx * xb[i], offc += idx * xc[i];
        }
        a.A = A + offa, a.B = B + offb, a.C = C + offc;
        /* a broadcast C dim outside the innermost: later passes accumulate onto the first */
        a.beta = (o > 0 && outer > 1 && offc == 0) ? 1.0f : beta;
        nck_gemm(nc__k(ctx), &a);
    }
}

static nc_status bmm_fwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    batch_dims bd;
    batch_shape(a, b, &bd);
    bmm_operand A, B;
    if (!bmm_operand_of(a, &bd, &A) || !bmm_operand_of(b, &bd, &B)) return NC_ERR_OOM;
    int64_t M = o->shape[bd.nb], N = o->shape[bd.nb + 1], K = a->shape[a->ndim - 1];
    int64_t sc[NC_MAX_DIMS];
    batch_strides(o, o->stride, &bd, sc);
    bmm_run(o->ctx, &bd, A.trans, B.trans, M, N, K, A.p, A.ld, A.bst, B.p, B.ld, B.bst, (float *)o->data, N, sc, 0.0f);
    return NC_OK;
}

static void bmm_bwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    nc_ctx *ctx = o->ctx;
    batch_dims bd;
    batch_shape(a, b, &bd);
    int64_t M = o->shape[bd.nb], N = o->shape[bd.nb + 1], K = a->shape[a->ndim - 1];
    const float *g = (const float *)o->grad->data;
    int64_t sg[NC_MAX_DIMS], cs[NC_MAX_DIMS], sgrad[NC_MAX_DIMS];
    nc__contig_strides(o->ndim, o->shape, cs);
    batch_strides(o, cs, &bd, sg);
    bmm_operand A, B;
    if (nc__needs_grad(a)) { /* dA_i += dC_i B_i^T */
        nc_tensor *ga = nc__grad_buf(a);
        if (ga && bmm_operand_of(b, &bd, &B)) {
            nc__contig_strides(a->ndim, a->shape, cs);
            batch_strides(a, cs, &bd, sgrad);
            bmm_run(ctx, &bd, 0, !B.trans, M, K, N, g, N, sg, B.p, B.ld, B.bst, (float *)ga->data, K, sgrad, 1.0f);
        }
    }
    if (nc__needs_grad(b)) { /* dB_i += A_i^T dC_i */
        nc_tensor *gb = nc__grad_buf(b);
        if (gb && bmm_operand_of(a, &bd, &A)) {
            nc__contig_strides(b->ndim, b->shape, cs);
            batch_strides(b, cs, &bd, sgrad);
            bmm_run(ctx, &bd, !A.trans, 0, K, N, M, A.p, A.ld, A.bst, g, N, sg, (float *)gb->data, N, sgrad, 1.0f);
        }
    }
}

const nc_op_def nc_op_bmm = {"bmm", 0, 0, bmm_infer, NULL, bmm_fwd, bmm_bwd};

nc_tensor *nc_matmul(nc_tensor *a, nc_tensor *b) {
    nc_tensor *in[2] = {a, b};
    return nc__apply(b && b->ndim > 2 ? &nc_op_bmm : &nc_op_matmul, in, 2, NULL);
}

/* ---- linear: y = x W^T + b ------------------------------------------------------------------------ */

static nc_status linear_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    for (int i = 0; i < n->n_in; i++)
        if (!nc__expect_f32(n, i)) return NC_ERR_DTYPE;
    if (x->ndim < 1 || w->ndim != 2 || x->shape[x->ndim - 1] != w->shape[1] ||
        (b && (b->ndim != 1 || b->shape[0] != w->shape[0]))) {
        char sx[96], sw[96], sb[96] = "none";
        if (b) nc__shape_str(b->ndim, b->shape, sb, sizeof sb);
        nc__error(x->ctx, NC_ERR_SHAPE, "linear: expected x [..., in], weight [out, in], bias [out]; got %s, %s, %s",
                  nc__shape_str(x->ndim, x->shape, sx, sizeof sx), nc__shape_str(w->ndim, w->shape, sw, sizeof sw), sb);
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    shape[x->ndim - 1] = w->shape[0];
    return NC_OK;
}

static nc_status linear_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    int64_t in = w->shape[1], out = w->shape[0], M = in ? nc_numel(x) / in : 0;
    const float *X = nc__contig_f32(x), *W = nc__contig_f32(w), *B = b ? nc__contig_f32(b) : NULL;
    if (!X || !W || (b && !B)) return NC_ERR_OOM;
    nck_gemm_args a;
    memset(&a, 0, sizeof a);
    a.ta = 0, a.tb = 1, a.M = M, a.N = out, a.K = in, a.alpha = 1.0f, a.beta = 0.0f;
    a.A = X, a.lda = in, a.B = W, a.ldb = in, a.C = (float *)n->out->data, a.ldc = out, a.batch = 1, a.bias = B;
    nck_gemm(nc__k(x->ctx), &a);
    return NC_OK;
}

static void linear_bwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    int64_t in = w->shape[1], out = w->shape[0], M = in ? nc_numel(x) / in : 0;
    const float *g = (const float *)n->out->grad->data;
    if (nc__needs_grad(x)) {
        const float *W = nc__contig_f32(w);
        int acc;
        nc_tensor *gx = W ? nc__grad_buf_acc(x, &acc) : NULL;
        if (gx && W) nc__gemm(x->ctx, 0, 0, M, in, out, 1.0f, g, out, W, in, acc ? 1.0f : 0.0f, (float *)gx->data, in);
    }
    if (nc__needs_grad(w)) {
        nc_tensor *gw = nc__grad_buf(w);
        const float *X = nc__contig_f32(x);
        if (gw && X) nc__gemm(x->ctx, 1, 0, out, in, M, 1.0f, g, out, X, in, 1.0f, (float *)gw->data, in);
    }
    if (b && nc__needs_grad(b)) {
        nc_tensor *gb = nc__grad_buf(b);
        if (gb) nck_colsum_acc(nc__k(x->ctx), g, (float *)gb->data, M, out);
    }
}

const nc_op_def nc_op_linear = {"linear", 0, 0, linear_infer, NULL, linear_fwd, linear_bwd};

nc_tensor *nc_linear_fn(nc_tensor *x, nc_tensor *weight, nc_tensor *bias) {
    nc_tensor *in[3] = {x, weight, bias};
    return nc__apply(&nc_op_linear, in, bias ? 3 : 2, NULL);
}
