/* Dense contractions: matmul (a [..., M, K] @ b [K, N], leading dims folded into M), batched matmul
 * with broadcast batch dims (b of rank > 2), and the fused linear layer y = x W^T + b. Shapes, the
 * dispatch between matmul and batched matmul, error messages and gradients are newch's
 * (engine/src/ops/ops_linalg.c: matmul :59-92, bmm :202-267, nc_matmul :269, linear :299-331).
 *
 * Everything is expressed with one abstraction: a strided matrix view (element (r, c) at
 * p[r * rs + c * cs]). A view with a unit column stride is a row-major GEMM operand, one with a unit
 * row stride a transposed one, so transposed tensors reach the tensor-core GEMM without a copy, and
 * every gradient is the forward contraction of transposed views (dA = dC B^T, dB = A^T dC). A view
 * with neither unit stride is materialised first. Batched products go through one planner that
 * merges batch dims wherever all three operands allow, runs the innermost as a strided-batch GEMM
 * launch and sums a broadcast output dim inside the launch (no atomics).
 */
#include "nc_internal.h"

typedef struct {
    const float *p;
    int64_t rs, cs; /* row and column strides, in elements */
} mat;

static mat mat_t(mat m) {
    mat t = {m.p, m.cs, m.rs};
    return t;
}

/* the GEMM operand form of a rows x cols view: 0 = row-major, 1 = transposed; -1 = neither */
static int gemm_form(mat m, int64_t rows, int64_t cols, int64_t *ld) {
    if (m.cs == 1 && m.rs >= cols) return *ld = m.rs, 0;
    if (m.rs == 1 && m.cs >= rows) return *ld = m.cs, 1;
    return -1;
}

/* The last two dims of t as a view usable by the GEMM (a contiguous copy when the strides do not
 * allow one). *bstride receives t's batch strides (of the copy when one was made). */
static int matrix_of(nc_tensor *t, mat *m, int64_t *bstride) {
    const int nd = t->ndim;
    const int64_t rows = t->shape[nd - 2], cols = t->shape[nd - 1];
    mat v = {NULL, t->stride[nd - 2], t->stride[nd - 1]};
    int64_t ld;
    if (gemm_form(v, rows, cols, &ld) >= 0) {
        v.p = (const float *)nc__dev(t);
        if (bstride) memcpy(bstride, t->stride, sizeof(int64_t) * (size_t)(nd - 2));
    } else {
        int64_t cst[NC_MAX_DIMS];
        nc__contig_strides(nd, t->shape, cst);
        v.p = nc__contig_f32(t);
        v.rs = cols, v.cs = 1;
        if (bstride) memcpy(bstride, cst, sizeof(int64_t) * (size_t)(nd - 2));
    }
    *m = v;
    return v.p != NULL;
}

static mat row_major(const float *p, int64_t ld) {
    mat m = {p, ld, 1};
    return m;
}

/* C = alpha A B + beta C (+ bias per column) for one product or a strided batch of them */
static void gemm_launch(nc_ctx *ctx, int64_t M, int64_t N, int64_t K, mat A, mat B, float *C, int64_t ldc, float beta,
                        const float *bias, int64_t batch, int64_t sA, int64_t sB, int64_t sC, int reduce) {
    nck_gemm_args g;
    memset(&g, 0, sizeof g);
    g.ta = gemm_form(A, M, K, &g.lda);
    g.tb = gemm_form(B, K, N, &g.ldb);
    g.M = M, g.N = N, g.K = K, g.alpha = 1.0f, g.beta = beta;
    g.A = A.p, g.B = B.p, g.C = C, g.ldc = ldc, g.bias = bias;
    g.batch = batch, g.sA = sA, g.sB = sB, g.sC = sC, g.reduce_batch = reduce;
    nck_gemm(nc__k(ctx), &g);
}

void nc__gemm(nc_ctx *ctx, int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
              const float *B, int64_t ldb, float beta, float *C, int64_t ldc) {
    nck_gemm_args g;
    memset(&g, 0, sizeof g);
    g.ta = ta, g.tb = tb, g.M = M, g.N = N, g.K = K, g.alpha = alpha, g.beta = beta;
    g.A = A, g.lda = lda, g.B = B, g.ldb = ldb, g.C = C, g.ldc = ldc, g.batch = 1;
    nck_gemm(nc__k(ctx), &g);
}

void nc__gemm_batched(nc_ctx *ctx, const nck_gemm_args *a) { nck_gemm(nc__k(ctx), a); }

/* ---- batched contraction planner -------------------------------------------------------------- */

typedef struct {
    int n;                                 /* batch dims after merging */
    int64_t ext[NC_MAX_DIMS];              /* their extents */
    int64_t st[3][NC_MAX_DIMS];            /* batch strides of A, B and C */
} batch_plan;

/* broadcast batch shape of two operands of ranks >= 2 (0 when they do not broadcast) */
static int broadcast_batch(const nc_tensor *a, const nc_tensor *b, int *nb, int64_t *ext) {
    const int na = a->ndim - 2, nbb = b->ndim - 2;
    *nb = na > nbb ? na : nbb;
    for (int i = 0; i < *nb; i++) {
        const int ia = i - (*nb - na), ib = i - (*nb - nbb);
        const int64_t da = ia >= 0 ? a->shape[ia] : 1, db = ib >= 0 ? b->shape[ib] : 1;
        if (da != db && da != 1 && db != 1) return 0;
        ext[i] = da == 1 ? db : da;
    }
    return 1;
}

/* t's stride along broadcast batch dim i (0 where t is broadcast), from its own batch strides */
static int64_t bstride_of(const nc_tensor *t, const int64_t *tst, int nb, int i) {
    const int j = i - (nb - (t->ndim - 2));
    return (j < 0 || t->shape[j] == 1) ? 0 : tst[j];
}

static void plan_batch(batch_plan *pl, int nb, const int64_t *ext, const nc_tensor *const t[3],
                       const int64_t *const tst[3]) {
    pl->n = 0;
    for (int i = 0; i < nb; i++) {
        if (ext[i] == 1) continue;
        int64_t s[3];
        for (int k = 0; k < 3; k++) s[k] = bstride_of(t[k], tst[k], nb, i);
        const int m = pl->n;
        /* dim i continues the previous one when every operand steps through both as one */
        if (m > 0 && pl->st[0][m - 1] == s[0] * ext[i] && pl->st[1][m - 1] == s[1] * ext[i] &&
            pl->st[2][m - 1] == s[2] * ext[i]) {
            pl->ext[m - 1] *= ext[i];
            for (int k = 0; k < 3; k++) pl->st[k][m - 1] = s[k];
            continue;
        }
        pl->ext[m] = ext[i];
        for (int k = 0; k < 3; k++) pl->st[k][m] = s[k];
        pl->n++;
    }
}

/* C_b (+)= A_b B_b over the plan: outer dims loop on the host, the innermost is one launch. A C slice
 * that an outer dim revisits (C broadcast there) accumulates after its first write. */
static void run_plan(nc_ctx *ctx, const batch_plan *pl, int64_t M, int64_t N, int64_t K, mat A, mat B, float *C,
                     int64_t ldc, float beta) {
    if (pl->n == 0) {
        gemm_launch(ctx, M, N, K, A, B, C, ldc, beta, NULL, 1, 0, 0, 0, 0);
        return;
    }
    const int last = pl->n - 1;
    int64_t outer = 1;
    for (int i = 0; i < last; i++) outer *= pl->ext[i];
    for (int64_t o = 0; o < outer; o++) {
        int64_t rem = o, off[3] = {0, 0, 0};
        int revisit = 0;
        for (int i = last - 1; i >= 0; i--) {
            const int64_t idx = rem % pl->ext[i];
            rem /= pl->ext[i];
            for (int k = 0; k < 3; k++) off[k] += idx * pl->st[k][i];
            if (idx > 0 && pl->st[2][i] == 0) revisit = 1;
        }
        mat Ao = {A.p + off[0], A.rs, A.cs}, Bo = {B.p + off[1], B.rs, B.cs};
        gemm_launch(ctx, M, N, K, Ao, Bo, C + off[2], ldc, revisit ? 1.0f : beta, NULL, pl->ext[last],
                    pl->st[0][last], pl->st[1][last], pl->st[2][last], pl->st[2][last] == 0);
    }
}

/* ---- matmul: a [..., M, K] @ b [K, N] ------------------------------------------------------------ */

static nc_status shape_error(nc_node *n, const char *expect) {
    const nc_tensor *a = n->in[0], *b = n->in[1];
    char sa[96], sb[96];
    nc__error(a->ctx, NC_ERR_SHAPE, "matmul: cannot multiply %s by %s (expected %s)",
              nc__shape_str(a->ndim, a->shape, sa, sizeof sa), nc__shape_str(b->ndim, b->shape, sb, sizeof sb), expect);
    return NC_ERR_SHAPE;
}

static nc_status matmul_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    const nc_tensor *a = n->in[0], *b = n->in[1];
    if (!nc__expect_f32(n, 0) || !nc__expect_f32(n, 1)) return NC_ERR_DTYPE;
    if (a->ndim < 2 || b->ndim != 2 || a->shape[a->ndim - 1] != b->shape[0])
        return shape_error(n, "[..., M, K] @ [K, N]");
    *dt = NC_F32;
    *nd = a->ndim;
    memcpy(shape, a->shape, sizeof(int64_t) * (size_t)a->ndim);
    shape[a->ndim - 1] = b->shape[1];
    return NC_OK;
}

/* a as an [M, K] view: a 2-d a keeps its strides, a folded one must be contiguous */
static int folded_lhs(nc_tensor *a, int64_t M, int64_t K, mat *m) {
    if (a->ndim == 2) return matrix_of(a, m, NULL);
    *m = row_major(nc__contig_f32(a), K);
    (void)M;
    return m->p != NULL;
}

static nc_status matmul_fwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    const int64_t K = b->shape[0], N = b->shape[1], M = nc_numel(a) / (K ? K : 1);
    mat A, B;
    if (!folded_lhs(a, M, K, &A) || !matrix_of(b, &B, NULL)) return NC_ERR_OOM;
    gemm_launch(n->out->ctx, M, N, K, A, B, (float *)n->out->data, N, 0.0f, NULL, 1, 0, 0, 0, 0);
    return NC_OK;
}

static void matmul_bwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    const int64_t K = b->shape[0], N = b->shape[1], M = nc_numel(a) / (K ? K : 1);
    const mat G = row_major((const float *)n->out->grad->data, N);
    int acc;
    mat A, B;
    if (nc__needs_grad(a) && matrix_of(b, &B, NULL)) { /* dA = dC B^T */
        nc_tensor *ga = nc__grad_buf_acc(a, &acc);
        if (ga) gemm_launch(a->ctx, M, K, N, G, mat_t(B), (float *)ga->data, K, acc ? 1.0f : 0.0f, NULL, 1, 0, 0, 0, 0);
    }
    if (nc__needs_grad(b) && folded_lhs(a, M, K, &A)) { /* dB = A^T dC */
        nc_tensor *gb = nc__grad_buf_acc(b, &acc);
        if (gb) gemm_launch(a->ctx, K, N, M, mat_t(A), G, (float *)gb->data, N, acc ? 1.0f : 0.0f, NULL, 1, 0, 0, 0, 0);
    }
}

const nc_op_def nc_op_matmul = {"matmul", 0, 0, matmul_infer, NULL, matmul_fwd, matmul_bwd};

/* ---- batched matmul: a [..., M, K] @ b [..., K, N] ------------------------------------------------ */

static nc_status bmm_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    const nc_tensor *a = n->in[0], *b = n->in[1];
    if (!nc__expect_f32(n, 0) || !nc__expect_f32(n, 1)) return NC_ERR_DTYPE;
    int nb = 0;
    int64_t ext[NC_MAX_DIMS];
    if (a->ndim < 2 || b->ndim < 2 || a->shape[a->ndim - 1] != b->shape[b->ndim - 2] || !broadcast_batch(a, b, &nb, ext))
        return shape_error(n, "[..., M, K] @ [..., K, N]");
    *dt = NC_F32;
    *nd = nb + 2;
    memcpy(shape, ext, sizeof(int64_t) * (size_t)nb);
    shape[nb] = a->shape[a->ndim - 2];
    shape[nb + 1] = b->shape[b->ndim - 1];
    return NC_OK;
}

typedef struct {
    int nb;
    int64_t ext[NC_MAX_DIMS];
    int64_t M, N, K;
} bmm_dims;

static void bmm_geometry(const nc_node *n, bmm_dims *d) {
    const nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    broadcast_batch(a, b, &d->nb, d->ext);
    d->M = o->shape[d->nb], d->N = o->shape[d->nb + 1], d->K = a->shape[a->ndim - 1];
}

static nc_status bmm_fwd(nc_node *n) {
    if (nc__attn_bmm(n)) return NC_OK; /* attention scores (a recipe) or probabilities @ v (fused) */
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    bmm_dims d;
    bmm_geometry(n, &d);
    mat A, B;
    int64_t sa[NC_MAX_DIMS], sb[NC_MAX_DIMS];
    if (!matrix_of(a, &A, sa) || !matrix_of(b, &B, sb)) return NC_ERR_OOM;
    const nc_tensor *ops[3] = {a, b, o};
    const int64_t *st[3] = {sa, sb, o->stride};
    batch_plan pl;
    plan_batch(&pl, d.nb, d.ext, ops, st);
    run_plan(o->ctx, &pl, d.M, d.N, d.K, A, B, (float *)o->data, d.N, 0.0f);
    return NC_OK;
}

static void bmm_bwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    bmm_dims d;
    bmm_geometry(n, &d);
    const mat G = row_major((const float *)o->grad->data, d.N);
    int64_t sg[NC_MAX_DIMS], sgrad[NC_MAX_DIMS], so[NC_MAX_DIMS];
    nc__contig_strides(o->ndim, o->shape, sg);
    mat X;
    batch_plan pl;
    if (nc__needs_grad(a)) { /* dA_i += dC_i B_i^T, summed over the dims where a is broadcast */
        nc_tensor *ga = nc__grad_buf(a);
        if (ga && matrix_of(b, &X, so)) {
            nc__contig_strides(a->ndim, a->shape, sgrad);
            const nc_tensor *ops[3] = {o, b, a};
            const int64_t *st[3] = {sg, so, sgrad};
            plan_batch(&pl, d.nb, d.ext, ops, st);
            run_plan(o->ctx, &pl, d.M, d.K, d.N, G, mat_t(X), (float *)ga->data, d.K, 1.0f);
        }
    }
    if (nc__needs_grad(b)) { /* dB_i += A_i^T dC_i */
        nc_tensor *gb = nc__grad_buf(b);
        if (gb && matrix_of(a, &X, so)) {
            nc__contig_strides(b->ndim, b->shape, sgrad);
            const nc_tensor *ops[3] = {a, o, b};
            const int64_t *st[3] = {so, sg, sgrad};
            plan_batch(&pl, d.nb, d.ext, ops, st);
            run_plan(o->ctx, &pl, d.K, d.N, d.M, mat_t(X), G, (float *)gb->data, d.N, 1.0f);
        }
    }
}

const nc_op_def nc_op_bmm = {"bmm", NC_OPF_RECIPE, 0, bmm_infer, NULL, bmm_fwd, bmm_bwd};

nc_tensor *nc_matmul(nc_tensor *a, nc_tensor *b) {
    nc_tensor *in[2] = {a, b};
    const nc_op_def *op = (b && b->ndim > 2) ? &nc_op_bmm : &nc_op_matmul;
    return nc__apply(op, in, 2, NULL);
}

/* ---- linear: y = x W^T + b ------------------------------------------------------------------------ */

static nc_status linear_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    const nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    for (int i = 0; i < n->n_in; i++)
        if (!nc__expect_f32(n, i)) return NC_ERR_DTYPE;
    const int ok = x->ndim >= 1 && w->ndim == 2 && x->shape[x->ndim - 1] == w->shape[1] &&
                   (!b || (b->ndim == 1 && b->shape[0] == w->shape[0]));
    if (!ok) {
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

typedef struct {
    int64_t in, out, rows;
} linear_dims;

static linear_dims linear_geometry(const nc_node *n) {
    const nc_tensor *x = n->in[0], *w = n->in[1];
    linear_dims d = {w->shape[1], w->shape[0], 0};
    d.rows = d.in ? nc_numel(x) / d.in : 0;
    return d;
}

static nc_status linear_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    const linear_dims d = linear_geometry(n);
    const float *X = nc__contig_f32(x), *W = nc__contig_f32(w), *bias = b ? nc__contig_f32(b) : NULL;
    if (!X || !W || (b && !bias)) return NC_ERR_OOM;
    /* y = X W^T: W's rows are the output features, so W^T is W read transposed; bias in the epilogue */
    gemm_launch(x->ctx, d.rows, d.out, d.in, row_major(X, d.in), mat_t(row_major(W, d.in)), (float *)n->out->data,
                d.out, 0.0f, bias, 1, 0, 0, 0, 0);
    return NC_OK;
}

static void linear_bwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    const linear_dims d = linear_geometry(n);
    const float *gy = (const float *)n->out->grad->data;
    const mat G = row_major(gy, d.out);
    if (nc__needs_grad(x)) { /* dX = dY W */
        const float *W = nc__contig_f32(w);
        int acc;
        nc_tensor *gx = W ? nc__grad_buf_acc(x, &acc) : NULL;
        if (gx)
            gemm_launch(x->ctx, d.rows, d.in, d.out, G, row_major(W, d.in), (float *)gx->data, d.in, acc ? 1.0f : 0.0f,
                        NULL, 1, 0, 0, 0, 0);
    }
    if (nc__needs_grad(w)) { /* dW += dY^T X (stored when the gradient is fresh: no fill, no read of C) */
        const float *X = nc__contig_f32(x);
        int acc = 1;
        nc_tensor *gw = X ? nc__grad_buf_acc(w, &acc) : NULL;
        if (gw)
            gemm_launch(x->ctx, d.out, d.in, d.rows, mat_t(G), row_major(X, d.in), (float *)gw->data, d.in,
                        acc ? 1.0f : 0.0f, NULL, 1, 0, 0, 0, 0);
    }
    if (b && nc__needs_grad(b)) { /* db += column sums of dY */
        nc_tensor *gb = nc__grad_buf(b);
        if (gb) nck_colsum_acc(nc__k(x->ctx), gy, (float *)gb->data, d.rows, d.out);
    }
}

const nc_op_def nc_op_linear = {"linear", 0, 0, linear_infer, NULL, linear_fwd, linear_bwd};

nc_tensor *nc_linear_fn(nc_tensor *x, nc_tensor *weight, nc_tensor *bias) {
    nc_tensor *in[3] = {x, weight, bias};
    return nc__apply(&nc_op_linear, in, bias ? 3 : 2, NULL);
}
