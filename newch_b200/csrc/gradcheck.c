/* Central-difference gradient check (newch engine/src/autograd/gradcheck.c:8-41): same error
 * measure |num - ana| / max(1, |num|, |ana|). Perturbations go through the inputs' host mirrors,
 * which reach the device before each re-evaluation; every evaluation waits for its loss. */
#include "nc_internal.h"

#include <math.h>
#include <stdlib.h>

float nc_gradcheck(nc_ctx *ctx, nc_scalar_fn fn, nc_tensor **inputs, int n_inputs, void *user, float eps) {
    for (int i = 0; i < n_inputs; i++) nc_zero_grad(inputs[i]);
    nc_tensor *y = fn(ctx, inputs, user);
    if (!y || nc_backward(y) != NC_OK) return INFINITY;
    float max_err = 0.0f;
    int prev = nc_set_grad_enabled(ctx, 0);
    for (int i = 0; i < n_inputs && nc_ok(ctx); i++) {
        nc_tensor *x = inputs[i];
        if (!nc__needs_grad(x)) continue;
        int64_t n = nc_numel(x);
        float *ana = (float *)calloc((size_t)(n ? n : 1), sizeof(float));
        if (!ana) break;
        if (x->grad) nc_copy_to(x->grad, ana, (size_t)n * sizeof(float));
        float *d = nc_data_f32(x);
        if (!d) {
            free(ana);
            nc__error(ctx, NC_ERR_ARG, "gradcheck: input %d must be contiguous f32", i);
            break;
        }
        for (int64_t j = 0; j < n; j++) {
            float orig = d[j];
            d[j] = orig + eps;
            float fp = nc_item(fn(ctx, inputs, user));
            d = nc_data_f32(x);
            d[j] = orig - eps;
            float fm = nc_item(fn(ctx, inputs, user));
            d = nc_data_f32(x);
            d[j] = orig;
            float num = (fp - fm) / (2.0f * eps);
            float a = ana[j];
            float denom = fmaxf(1.0f, fmaxf(fabsf(num), fabsf(a)));
            float err = fabsf(num - a) / denom;
            if (!(err <= max_err)) max_err = err;
        }
        nc__dev(x);
        free(ana);
    }
    nc_set_grad_enabled(ctx, prev);
    return nc_ok(ctx) ? max_err : INFINITY;
}
