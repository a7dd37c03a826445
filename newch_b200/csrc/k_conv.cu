// Convolution and pooling kernels (NCHW): batched im2col / gather-form col2im, per-channel bias
// gradients, direct convolution for few input channels, depthwise forward / dX / dW, pooling.
//
// Index conventions are newch's (engine/src/ops/ops_conv.c: im2col rows ordered (c, ki, kj) with
// columns (oy, ox) :66-86; depthwise :192-283; pooling with a window-local first maximum and
// count_include_pad averaging :434-509). Gradients that several outputs feed are gathered per
// destination element in a fixed order instead of scattered with atomics.
#include "k_common.cuh"

using namespace nck;

// col[n - n0][c * KH * KW + ki * KW + kj][oy * OW + ox] for samples n0 .. n0 + nb
__global__ void k_im2col(nck_conv g, const float *__restrict__ x, float *__restrict__ col, int64_t n0, int64_t nb) {
    int64_t L = g.OH * g.OW, KK = g.KH * g.KW, rows = g.C * KK;
    int64_t total = nb * rows * L;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t l = t % L, rr = t / L;
        int64_t row = rr % rows, n = rr / rows + n0;
        int64_t c = row / KK, kk = row - c * KK, ki = kk / g.KW, kj = kk - ki * g.KW;
        int64_t oy = l / g.OW, ox = l - oy * g.OW;
        int64_t iy = oy * g.sh - g.ph + ki * g.dh, ix = ox * g.sw - g.pw + kj * g.dw;
        float v = 0.0f;
        if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W) v = x[((n * g.C + c) * g.H + iy) * g.W + ix];
        col[t] = v;
    }
}

extern "C" void nck_im2col(nck_dev *d, const nck_conv *g, const float *x, float *col, int64_t n0, int64_t nb) {
    int64_t total = nb * g->C * g->KH * g->KW * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, "im2col", 0.0, 4.0 * (nb * g->C * g->H * g->W + total));
    k_im2col<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, x, col, n0, nb);
    NCK_LAUNCHED(d, 1);
}

// dx[n, c, iy, ix] += sum over (ki, kj) hitting it of col[n][c, ki, kj][oy, ox]
__global__ void k_col2im(nck_conv g, const float *__restrict__ col, float *__restrict__ dx, int64_t n0, int64_t nb) {
    int64_t L = g.OH * g.OW, KK = g.KH * g.KW;
    int64_t total = nb * g.C * g.H * g.W;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ix = t % g.W, r = t / g.W;
        int64_t iy = r % g.H;
        r /= g.H;
        int64_t c = r % g.C, n = r / g.C;
        const float *cb = col + (n * g.C + c) * KK * L;
        float acc = 0.0f;
        for (int64_t ki = 0; ki < g.KH; ki++) {
            int64_t ty = iy + g.ph - ki * g.dh;
            if (ty < 0 || ty % g.sh) continue;
            int64_t oy = ty / g.sh;
            if (oy >= g.OH) continue;
            for (int64_t kj = 0; kj < g.KW; kj++) {
                int64_t tx = ix + g.pw - kj * g.dw;
                if (tx < 0 || tx % g.sw) continue;
                int64_t ox = tx / g.sw;
                if (ox >= g.OW) continue;
                acc += cb[(ki * g.KW + kj) * L + oy * g.OW + ox];
            }
        }
        dx[((n + n0) * g.C + c) * g.H * g.W + iy * g.W + ix] += acc;
    }
}

extern "C" void nck_col2im(nck_dev *d, const nck_conv *g, const float *col, float *dx, int64_t n0, int64_t nb) {
    int64_t total = nb * g->C * g->H * g->W;
    if (total <= 0) return;
    Scope sc(d, "col2im", 0.0, 4.0 * (nb * g->C * g->KH * g->KW * g->OH * g->OW + 2 * total));
    k_col2im<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, col, dx, n0, nb);
    NCK_LAUNCHED(d, 1);
}

// ---- per-channel sums over [N, C, S] (bias gradients) -----------------------------------------------

__global__ void k_chan_sum_partial(const float *__restrict__ x, float *__restrict__ part, int64_t N, int64_t C,
                                   int64_t S, int64_t per_split) {
    __shared__ float sm[kThreads / 32];
    int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    float acc = 0.0f;
    for (int64_t n = n0; n < n1; n++) {
        const float *p = x + (n * C + c) * S;
        for (int64_t j = threadIdx.x; j < S; j += blockDim.x) acc += p[j];
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) s += sm[k];
        part[blockIdx.y * C + c] = s;
    }
}

__global__ void k_chan_sum_combine(const float *__restrict__ part, int splits, int64_t C, float *__restrict__ gb) {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < C; c += (int64_t)gridDim.x * blockDim.x) {
        float s = gb[c];
        for (int k = 0; k < splits; k++) s += part[k * C + c];
        gb[c] = s;
    }
}

extern "C" void nck_conv_bias_grad(nck_dev *d, const float *g, float *gb, int64_t N, int64_t OC, int64_t L) {
    if (N * OC * L <= 0) return;
    Scope sc(d, "conv_bias_grad");
    int64_t splits = ((int64_t)d->sm_count * 4 + OC - 1) / OC;
    if (splits > N) splits = N;
    if (splits < 1) splits = 1;
    int64_t per = (N + splits - 1) / splits;
    splits = (N + per - 1) / per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)OC, (unsigned)splits);
    k_chan_sum_partial<<<grid, kThreads, 0, NCK_STREAM(d)>>>(g, part, N, OC, L, per);
    k_chan_sum_combine<<<grid_for(d, OC), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, OC, gb);
    NCK_LAUNCHED(d, 2);
}

// ---- direct convolution: each thread reads its receptive field once and produces every output
// channel of its group at that position (Cg * KH * KW <= 32, OCg <= 64) ---------------------------------

__global__ void k_conv_direct(nck_conv g, const float *__restrict__ x, const float *__restrict__ w,
                              const float *__restrict__ b, float *__restrict__ y) {
    __shared__ float ws[64 * 32];
    int64_t Cg = g.C / g.G, OCg = g.OC / g.G, KK = g.KH * g.KW, CKK = Cg * KK, L = g.OH * g.OW;
    int64_t ng = blockIdx.y;  // (n, group)
    int64_t n = ng / g.G, gi = ng % g.G;
    for (int64_t i = threadIdx.x; i < OCg * CKK; i += blockDim.x) ws[i] = w[gi * OCg * CKK + i];
    __syncthreads();
    for (int64_t l = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; l < L; l += (int64_t)gridDim.x * blockDim.x) {
        int64_t oy = l / g.OW, ox = l - oy * g.OW;
        float in[32];
        for (int64_t k = 0; k < CKK; k++) {
            int64_t c = k / KK, kk = k - c * KK, ki = kk / g.KW, kj = kk - ki * g.KW;
            int64_t iy = oy * g.sh - g.ph + ki * g.dh, ix = ox * g.sw - g.pw + kj * g.dw;
            in[k] = (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W)
                        ? x[((n * g.C + gi * Cg + c) * g.H + iy) * g.W + ix]
                        : 0.0f;
        }
        for (int64_t o = 0; o < OCg; o++) {
            float acc = b ? b[gi * OCg + o] : 0.0f;
            for (int64_t k = 0; k < CKK; k++) acc = fmaf(ws[o * CKK + k], in[k], acc);
            y[(n * g.OC + gi * OCg + o) * L + l] = acc;
        }
    }
}

extern "C" void nck_conv_direct_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b,
                                    float *y) {
    int64_t L = g->OH * g->OW;
    if (g->N * g->G * L <= 0) return;
    Scope sc(d, "conv_direct", 2.0 * g->N * g->OC * L * (g->C / g->G) * g->KH * g->KW,
             4.0 * (g->N * g->C * g->H * g->W + g->N * g->OC * L));
    int64_t bx = (L + kThreads - 1) / kThreads;
    if (bx > 64) bx = 64;
    dim3 grid((unsigned)bx, (unsigned)(g->N * g->G));
    k_conv_direct<<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, w, b, y);
    NCK_LAUNCHED(d, 1);
}

// ---- depthwise (groups == C == OC) ---------------------------------------------------------------

// y = bias + sum over (ki, kj) in order of w * x, fused multiply-adds as newch's axpy rows
__global__ void k_dw_fwd(nck_conv g, const float *__restrict__ x, const float *__restrict__ w,
                         const float *__restrict__ b, float *__restrict__ y) {
    int64_t total = g.N * g.C * g.OH * g.OW;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ox = t % g.OW, r = t / g.OW;
        int64_t oy = r % g.OH, plane = r / g.OH;
        int64_t c = plane % g.C;
        const float *xp = x + plane * g.H * g.W, *wk = w + c * g.KH * g.KW;
        float acc = b ? b[c] : 0.0f;
        for (int64_t ki = 0; ki < g.KH; ki++) {
            int64_t iy = oy * g.sh - g.ph + ki * g.dh;
            if (iy < 0 || iy >= g.H) continue;
            for (int64_t kj = 0; kj < g.KW; kj++) {
                int64_t ix = ox * g.sw - g.pw + kj * g.dw;
                if (ix < 0 || ix >= g.W) continue;
                acc = fmaf(wk[ki * g.KW + kj], xp[iy * g.W + ix], acc);
            }
        }
        y[t] = acc;
    }
}

extern "C" void nck_dw_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b, float *y) {
    int64_t total = g->N * g->C * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, "dw_fwd", 2.0 * total * g->KH * g->KW, 4.0 * (g->N * g->C * g->H * g->W + total));
    k_dw_fwd<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, x, w, b, y);
    NCK_LAUNCHED(d, 1);
}

// dx[n, c, iy, ix] += sum over taps reaching it of w * gy
__global__ void k_dw_dx(nck_conv g, const float *__restrict__ gy, const float *__restrict__ w, float *__restrict__ gx) {
    int64_t total = g.N * g.C * g.H * g.W;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ix = t % g.W, r = t / g.W;
        int64_t iy = r % g.H, plane = r / g.H;
        int64_t c = plane % g.C;
        const float *gp = gy + plane * g.OH * g.OW, *wk = w + c * g.KH * g.KW;
        float acc = gx[t];
        for (int64_t ki = 0; ki < g.KH; ki++) {
            int64_t ty = iy + g.ph - ki * g.dh;
            if (ty < 0 || ty % g.sh) continue;
            int64_t oy = ty / g.sh;
            if (oy >= g.OH) continue;
            for (int64_t kj = 0; kj < g.KW; kj++) {
                int64_t tx = ix + g.pw - kj * g.dw;
                if (tx < 0 || tx % g.sw) continue;
                int64_t ox = tx / g.sw;
                if (ox >= g.OW) continue;
                acc = fmaf(wk[ki * g.KW + kj], gp[oy * g.OW + ox], acc);
            }
        }
        gx[t] = acc;
    }
}

extern "C" void nck_dw_dx(nck_dev *d, const nck_conv *g, const float *gy, const float *w, float *gx) {
    int64_t total = g->N * g->C * g->H * g->W;
    if (total <= 0) return;
    Scope sc(d, "dw_dx", 2.0 * g->N * g->C * g->OH * g->OW * g->KH * g->KW,
             4.0 * (g->N * g->C * g->OH * g->OW + 2 * total));
    k_dw_dx<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, w, gx);
    NCK_LAUNCHED(d, 1);
}

// weight grads: per channel, per tap, the sum over samples and output positions of x * gy;
// grid (C, splits over N), at most NCK_DW_MAX_TAPS taps, partials combined in order
__global__ void k_dw_dw_partial(nck_conv g, const float *__restrict__ x, const float *__restrict__ gy,
                                float *__restrict__ part, int64_t per_split) {
    __shared__ float sm[kThreads / 32][NCK_DW_MAX_TAPS];
    int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < g.N ? n0 + per_split : g.N;
    int KK = (int)(g.KH * g.KW);
    float acc[NCK_DW_MAX_TAPS];
    for (int k = 0; k < NCK_DW_MAX_TAPS; k++) acc[k] = 0.0f;
    int64_t L = g.OH * g.OW;
    for (int64_t n = n0; n < n1; n++) {
        const float *xp = x + (n * g.C + c) * g.H * g.W, *gp = gy + (n * g.C + c) * L;
        for (int64_t l = threadIdx.x; l < L; l += blockDim.x) {
            int64_t oy = l / g.OW, ox = l - oy * g.OW;
            float gv = gp[l];
            for (int k = 0; k < KK; k++) {
                int64_t ki = k / g.KW, kj = k - ki * g.KW;
                int64_t iy = oy * g.sh - g.ph + ki * g.dh, ix = ox * g.sw - g.pw + kj * g.dw;
                if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W) acc[k] = fmaf(xp[iy * g.W + ix], gv, acc[k]);
            }
        }
    }
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int k = 0; k < KK; k++) {
        float v = acc[k];
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sm[wid][k] = v;
    }
    __syncthreads();
    if (threadIdx.x < KK) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += sm[w][threadIdx.x];
        part[(blockIdx.y * g.C + c) * KK + threadIdx.x] = s;
    }
}

__global__ void k_dw_dw_combine(const float *__restrict__ part, int splits, int64_t C, int KK, float *__restrict__ gw) {
    int64_t total = C * KK;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        float s = gw[t];
        for (int k = 0; k < splits; k++) s += part[k * total + t];
        gw[t] = s;
    }
}

extern "C" void nck_dw_dw(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb) {
    (void)gb; /* the bias gradient goes through nck_conv_bias_grad */
    int KK = (int)(g->KH * g->KW);
    if (g->N * g->C <= 0 || KK <= 0) return;
    if (KK > NCK_DW_MAX_TAPS) return; /* the caller takes the im2col path for larger kernels */
    Scope sc(d, "dw_dw", 2.0 * g->N * g->C * g->OH * g->OW * KK,
             4.0 * (g->N * g->C * (g->H * g->W + g->OH * g->OW)));
    int64_t splits = ((int64_t)d->sm_count * 4 + g->C - 1) / g->C;
    if (splits > g->N) splits = g->N;
    if (splits < 1) splits = 1;
    int64_t per = (g->N + splits - 1) / splits;
    splits = (g->N + per - 1) / per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)g->C, (unsigned)splits);
    k_dw_dw_partial<<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, gy, part, per);
    k_dw_dw_combine<<<grid_for(d, g->C * KK), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, g->C, KK, gw);
    NCK_LAUNCHED(d, 2);
}

// ---- pooling ---------------------------------------------------------------------------------------------

__global__ void k_pool_fwd(nck_conv g, const float *__restrict__ x, float *__restrict__ y, int32_t *__restrict__ arg,
                           int is_max) {
    int64_t total = g.N * g.C * g.OH * g.OW;
    float inv = 1.0f / (float)(g.KH * g.KW);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ox = t % g.OW, r = t / g.OW;
        int64_t oy = r % g.OH, plane = r / g.OH;
        const float *xp = x + plane * g.H * g.W;
        float best = -INFINITY, acc = 0.0f;
        int32_t bi = -1;
        for (int64_t ki = 0; ki < g.KH; ki++) {
            int64_t iy = oy * g.sh - g.ph + ki;
            if (iy < 0 || iy >= g.H) continue;
            for (int64_t kj = 0; kj < g.KW; kj++) {
                int64_t ix = ox * g.sw - g.pw + kj;
                if (ix < 0 || ix >= g.W) continue;
                float v = xp[iy * g.W + ix];
                acc += v;
                if (v > best || bi < 0) best = v, bi = (int32_t)(iy * g.W + ix);
            }
        }
        if (is_max) {
            y[t] = best;
            arg[t] = bi;
        } else {
            y[t] = acc * inv;
        }
    }
}

extern "C" void nck_pool_fwd(nck_dev *d, const nck_conv *g, const float *x, float *y, int32_t *arg, int is_max) {
    int64_t total = g->N * g->C * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, is_max ? "max_pool" : "avg_pool", 0.0,
             4.0 * (g->N * g->C * g->H * g->W + (is_max ? 2 : 1) * total));
    k_pool_fwd<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, x, y, arg, is_max);
    NCK_LAUNCHED(d, 1);
}

// windows that do not overlap: each output adds its gradient to the one input it came from
__global__ void k_maxpool_bwd_scatter(nck_conv g, const float *__restrict__ gy, const int32_t *__restrict__ arg,
                                      float *__restrict__ gx) {
    int64_t per = g.OH * g.OW, total = g.N * g.C * per;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x)
        gx[(t / per) * g.H * g.W + arg[t]] += gy[t];
}

// general windows: each input gathers from the outputs whose window holds it, in output order
__global__ void k_pool_bwd_gather(nck_conv g, const float *__restrict__ gy, const int32_t *__restrict__ arg,
                                  float *__restrict__ gx, int is_max) {
    int64_t total = g.N * g.C * g.H * g.W;
    float inv = 1.0f / (float)(g.KH * g.KW);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ix = t % g.W, r = t / g.W;
        int64_t iy = r % g.H, plane = r / g.H;
        int32_t self = (int32_t)(iy * g.W + ix);
        const float *gp = gy + plane * g.OH * g.OW;
        const int32_t *ap = is_max ? arg + plane * g.OH * g.OW : nullptr;
        float acc = gx[t];
        int64_t oy0 = iy + g.ph - (g.KH - 1);
        oy0 = oy0 <= 0 ? 0 : (oy0 + g.sh - 1) / g.sh;
        int64_t oy1 = (iy + g.ph) / g.sh;
        int64_t ox0 = ix + g.pw - (g.KW - 1);
        ox0 = ox0 <= 0 ? 0 : (ox0 + g.sw - 1) / g.sw;
        int64_t ox1 = (ix + g.pw) / g.sw;
        for (int64_t oy = oy0; oy <= oy1 && oy < g.OH; oy++)
            for (int64_t ox = ox0; ox <= ox1 && ox < g.OW; ox++) {
                int64_t o = oy * g.OW + ox;
                if (is_max) {
                    if (ap[o] == self) acc += gp[o];
                } else {
                    acc += gp[o] * inv;
                }
            }
        gx[t] = acc;
    }
}

extern "C" void nck_pool_bwd(nck_dev *d, const nck_conv *g, const float *gy, const int32_t *arg, float *gx,
                             int is_max) {
    Scope sc(d, is_max ? "max_pool_bwd" : "avg_pool_bwd", 0.0,
             4.0 * ((is_max ? 2 : 1) * g->N * g->C * g->OH * g->OW + 2 * g->N * g->C * g->H * g->W));
    if (is_max && g->sh >= g->KH && g->sw >= g->KW) {
        int64_t total = g->N * g->C * g->OH * g->OW;
        if (total <= 0) return;
        k_maxpool_bwd_scatter<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx);
    } else {
        int64_t total = g->N * g->C * g->H * g->W;
        if (total <= 0) return;
        k_pool_bwd_gather<<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx, is_max);
    }
    NCK_LAUNCHED(d, 1);
}
