/* nc_gradcheck: compares the autograd gradient of a scalar function with central differences.
 *
 * The result is newch's (engine/src/autograd/gradcheck.c:8-41): for every element of every input
 * that requires grad, num = (f(x + eps) - f(x - eps)) / (2 eps), and the largest
 * |num - ana| / max(1, |num|, |ana|) is returned (INFINITY when the context failed).
 *
 * On the device the inputs stay where they are: each probe writes one element (4 bytes, from a host
 * snapshot of the input taken once) straight into device memory, evaluates, and writes the next;
 * the whole input is never copied back and forth per element.
 */
#include "nc_internal.h"

#include <math.h>
#include <stdlib.h>

/* device address of element j of a contiguous f32 input, after pending host writes are flushed */
static float *element_addr(nc_tensor *x, int64_t j) { return (float *)nc__dev(x) + j; }

static void poke(nc_ctx *ctx, nc_tensor *x, int64_t j, float v) {
    nc__upload(ctx, element_addr(x, j), &v, sizeof v);
    nc__dev_write(x); /* a host mirror of x no longer matches */
}

static float probe(nc_ctx *ctx, nc_scalar_fn fn, nc_tensor **inputs, void *user) {
    nc_tensor *y = fn(ctx, inputs, user);
    return y ? nc_item(y) : NAN;
}

static float check_input(nc_ctx *ctx, nc_scalar_fn fn, nc_tensor **inputs, int i, void *user, float eps) {
    nc_tensor *x = inputs[i];
    const int64_t n = nc_numel(x);
    if (x->dtype != NC_F32 || !nc_is_contiguous(x)) {
        nc__error(ctx, NC_ERR_ARG, "gradcheck: input %d must be contiguous f32", i);
        return INFINITY;
    }
    float *base = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    float *ana = (float *)calloc((size_t)(n > 0 ? n : 1), sizeof(float));
    if (!base || !ana) {
        free(base);
        free(ana);
        nc__error(ctx, NC_ERR_OOM, "gradcheck: out of host memory");
        return INFINITY;
    }
    float worst = 0.0f;
    if (nc_copy_to(x, base, sizeof(float) * (size_t)n) && (!x->grad || nc_copy_to(x->grad, ana, sizeof(float) * (size_t)n))) {
        for (int64_t j = 0; j < n && nc_ok(ctx); j++) {
            poke(ctx, x, j, base[j] + eps);
            const float fp = probe(ctx, fn, inputs, user);
            poke(ctx, x, j, base[j] - eps);
            const float fm = probe(ctx, fn, inputs, user);
            poke(ctx, x, j, base[j]);
            const float num = (fp - fm) / (2.0f * eps);
            const float scale = fmaxf(1.0f, fmaxf(fabsf(num), fabsf(ana[j])));
            const float err = fabsf(num - ana[j]) / scale;
            if (!(err <= worst)) worst = err; /* a NaN error sticks */
        }
    }
    free(base);
    free(ana);
    return worst;
}

float nc_gradcheck(nc_ctx *ctx, nc_scalar_fn fn, nc_tensor **inputs, int n_inputs, void *user, float eps) {
    for (int i = 0; i < n_inputs; i++) nc_zero_grad(inputs[i]);
    nc_tensor *y = fn(ctx, inputs, user);
    if (!y || nc_backward(y) != NC_OK) return INFINITY;
    const int grad_was = nc_set_grad_enabled(ctx, 0);
    float worst = 0.0f;
    for (int i = 0; i < n_inputs && nc_ok(ctx); i++) {
        if (!nc__needs_grad(inputs[i])) continue;
        const float e = check_input(ctx, fn, inputs, i, user, eps);
        if (!(e <= worst)) worst = e;
    }
    nc_set_grad_enabled(ctx, grad_was);
    return nc_ok(ctx) ? worst : INFINITY;
}
