/* C modules for programs that build models without Python: Linear, an activation, Sequential.
 *
 * newch's C API (engine/include/nc.h nc_linear / nc_act / nc_sequential / nc_forward /
 * nc_parameters / nc_set_training / nc_module_name) is kept; underneath, a module here is one tagged
 * record interpreted by a single dispatcher rather than a per-type function table. Linear keeps
 * newch's initialisation, which its users' seeds depend on: weight, then bias, each element drawn in
 * order from the context's stream as bound * (2u - 1) with bound = 1 / sqrt(in_features)
 * (engine/src/nn/modules.c:55-78). The draws are made on the host (the stream is host-authoritative)
 * and uploaded once. Records live in the context's persistent host memory, freed with it.
 */
#include "nc_internal.h"

#include <math.h>
#include <stdlib.h>

typedef enum { MOD_LINEAR, MOD_ACTIVATION, MOD_SEQUENCE } mod_kind;

struct nc_module {
    mod_kind kind;
    nc_ctx *ctx;
    int training;
    union {
        struct {
            nc_tensor *weight, *bias; /* bias may be NULL */
        } linear;
        nc_activation activation;
        struct {
            int count;
            nc_module **items;
        } sequence;
    } u;
};

static nc_module *module_new(nc_ctx *ctx, mod_kind kind) {
    nc_module *m = (nc_module *)nc__meta_alloc(ctx, sizeof(nc_module), 1);
    if (!m) return NULL;
    memset(m, 0, sizeof *m);
    m->kind = kind;
    m->ctx = ctx;
    m->training = 1;
    return m;
}

/* a new parameter of `shape` holding U(-bound, bound) draws from the context stream */
static nc_tensor *uniform_parameter(nc_ctx *ctx, int ndim, const int64_t *shape, float bound, const char *name) {
    nc_tensor *p = nc_parameter(ctx, NULL, ndim, shape);
    if (!p) return NULL;
    nc_set_name(p, name);
    const int64_t n = nc_numel(p);
    float *vals = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    if (!vals) {
        nc__error(ctx, NC_ERR_OOM, "out of host memory");
        return NULL;
    }
    for (int64_t i = 0; i < n; i++) {
        const float u = nc__rand_uniform01(ctx);
        vals[i] = bound * (2.0f * u - 1.0f);
    }
    const int ok = nc_copy_from(p, vals, sizeof(float) * (size_t)n);
    free(vals);
    return ok ? p : NULL;
}

nc_module *nc_linear(nc_ctx *ctx, int64_t in_features, int64_t out_features, int bias) {
    if (in_features <= 0 || out_features <= 0) {
        nc__error(ctx, NC_ERR_ARG, "linear: features must be positive");
        return NULL;
    }
    nc_module *m = module_new(ctx, MOD_LINEAR);
    if (!m) return NULL;
    const float bound = 1.0f / sqrtf((float)in_features);
    const int64_t wshape[2] = {out_features, in_features};
    m->u.linear.weight = uniform_parameter(ctx, 2, wshape, bound, "weight");
    if (!m->u.linear.weight) return NULL;
    if (bias && !(m->u.linear.bias = uniform_parameter(ctx, 1, &out_features, bound, "bias"))) return NULL;
    return m;
}

nc_module *nc_act(nc_ctx *ctx, nc_activation kind) {
    if (kind != NC_ACT_RELU && kind != NC_ACT_SIGMOID && kind != NC_ACT_TANH) {
        nc__error(ctx, NC_ERR_ARG, "act: unknown activation %d", (int)kind);
        return NULL;
    }
    nc_module *m = module_new(ctx, MOD_ACTIVATION);
    if (m) m->u.activation = kind;
    return m;
}

nc_module *nc_sequential(nc_ctx *ctx, int n, nc_module **mods) {
    for (int i = 0; i < n; i++)
        if (!mods[i]) return NULL; /* a failed constructor upstream */
    nc_module *m = module_new(ctx, MOD_SEQUENCE);
    nc_module **items = (nc_module **)nc__meta_alloc(ctx, sizeof(nc_module *) * (size_t)(n > 0 ? n : 1), 1);
    if (!m || !items) return NULL;
    if (n > 0) memcpy(items, mods, sizeof(nc_module *) * (size_t)n);
    m->u.sequence.count = n;
    m->u.sequence.items = items;
    return m;
}

nc_tensor *nc_forward(nc_module *m, nc_tensor *x) {
    if (!m || !x) return NULL;
    switch (m->kind) {
    case MOD_LINEAR: return nc_linear_fn(x, m->u.linear.weight, m->u.linear.bias);
    case MOD_ACTIVATION:
        return m->u.activation == NC_ACT_RELU ? nc_relu(x) : m->u.activation == NC_ACT_SIGMOID ? nc_sigmoid(x) : nc_tanh(x);
    case MOD_SEQUENCE:
        for (int i = 0; i < m->u.sequence.count && x; i++) x = nc_forward(m->u.sequence.items[i], x);
        return x;
    }
    return NULL;
}

/* Depth-first parameter walk: writes up to `max` tensors to out and returns how many exist. */
static int collect_params(const nc_module *m, nc_tensor **out, int max, int found) {
    switch (m->kind) {
    case MOD_LINEAR: {
        nc_tensor *ps[2] = {m->u.linear.weight, m->u.linear.bias};
        for (int k = 0; k < 2; k++) {
            if (!ps[k]) continue;
            if (out && found < max) out[found] = ps[k];
            found++;
        }
        return found;
    }
    case MOD_SEQUENCE:
        for (int i = 0; i < m->u.sequence.count; i++) found = collect_params(m->u.sequence.items[i], out, max, found);
        return found;
    case MOD_ACTIVATION: return found;
    }
    return found;
}

int nc_parameters(nc_module *m, nc_tensor **out, int max) { return m ? collect_params(m, out, max, 0) : 0; }

const char *nc_module_name(const nc_module *m) {
    if (!m) return "";
    switch (m->kind) {
    case MOD_LINEAR: return "Linear";
    case MOD_SEQUENCE: return "Sequential";
    case MOD_ACTIVATION:
        return m->u.activation == NC_ACT_RELU ? "ReLU" : m->u.activation == NC_ACT_SIGMOID ? "Sigmoid" : "Tanh";
    }
    return "";
}

void nc_set_training(nc_module *m, int training) {
    if (!m) return;
    m->training = training ? 1 : 0;
    if (m->kind == MOD_SEQUENCE)
        for (int i = 0; i < m->u.sequence.count; i++) nc_set_training(m->u.sequence.items[i], training);
}
