// Convolution and pooling kernels (NCHW): batched im2col / gather-form col2im, per-channel bias
// gradients, direct convolution for few input channels, depthwise forward / dX / dW, pooling.
//
// Index conventions are newch's (engine/src/ops/ops_conv.c: im2col rows ordered (c, ki, kj) with
// columns (oy, ox) :66-86; depthwise :192-283; pooling with a window-local first maximum and
// count_include_pad averaging :434-509). Gradients that several outputs feed are gathered per
// destination element in a fixed order instead of scattered with atomics.
#include "k_common.cuh"

using namespace nck;

// Unfold and fold run one (sample, channel) plane per block: index arithmetic inside a plane is 32-bit
// (a plane is far below 2^31 elements), each thread owns output positions of the plane, and for a
// fixed tap the threads of a warp touch consecutive addresses.

// col[n - n0][c * KH * KW + ki * KW + kj][oy * OW + ox] for samples n0 .. n0 + nb
__global__ void __launch_bounds__(128) k_im2col(nck_conv g, const float *__restrict__ x, float *__restrict__ col,
                                                int64_t n0, int64_t nb) {
    const int L = (int)(g.OH * g.OW), OW = (int)g.OW, H = (int)g.H, W = (int)g.W;
    const int KH = (int)g.KH, KW = (int)g.KW, KK = KH * KW;
    const int64_t planes = nb * g.C;
    for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
        const float *xp = x + (n0 * g.C + pl) * (int64_t)H * W;  // planes of samples n0.. are consecutive
        float *cp = col + pl * (int64_t)KK * L;
        for (int l = threadIdx.x; l < L; l += blockDim.x) {
            int oy = l / OW, ox = l - oy * OW;
            int iy0 = oy * g.sh - g.ph, ix0 = ox * g.sw - g.pw;
            for (int ki = 0; ki < KH; ki++) {
                int iy = iy0 + ki * g.dh;
                bool rowok = iy >= 0 && iy < H;
                for (int kj = 0; kj < KW; kj++) {
                    int ix = ix0 + kj * g.dw;
                    float v = (rowok && ix >= 0 && ix < W) ? __ldg(xp + iy * W + ix) : 0.0f;
                    cp[(ki * KW + kj) * L + l] = v;
                }
            }
        }
    }
}

static int plane_grid(const nck_dev *d, int64_t planes) {
    int64_t cap = (int64_t)(d->sm_count > 0 ? d->sm_count : 148) * 16;
    return (int)(planes < cap ? (planes > 0 ? planes : 1) : cap);
}

extern "C" void nck_im2col(nck_dev *d, const nck_conv *g, const float *x, float *col, int64_t n0, int64_t nb) {
    int64_t total = nb * g->C * g->KH * g->KW * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, "im2col", 0.0, 4.0 * (nb * g->C * g->H * g->W + total));
    k_im2col<<<plane_grid(d, nb * g->C), 128, 0, NCK_STREAM(d)>>>(*g, x, col, n0, nb);
    NCK_LAUNCHED(d, 1);
}

// dx[n, c, iy, ix] += sum over the taps (ki, kj) whose window covers it of col[n][c, ki, kj][oy, ox],
// taps in (ki, kj) order. STAGE: the plane's contiguous KH*KW*L slab of col is first copied to shared
// memory with 16-byte loads (full-bandwidth reads), and the gathers read shared memory.
template <bool STAGE>
__global__ void __launch_bounds__(256) k_col2im(nck_conv g, const float *__restrict__ col, float *__restrict__ dx,
                                                int64_t n0, int64_t nb, int accum) {
    extern __shared__ float slab[];
    const int L = (int)(g.OH * g.OW), OH = (int)g.OH, OW = (int)g.OW, H = (int)g.H, W = (int)g.W;
    const int KH = (int)g.KH, KW = (int)g.KW, KK = KH * KW, HW = H * W;
    const int64_t planes = nb * g.C;
    for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
        const float *cb = col + pl * (int64_t)KK * L;
        float *dp = dx + (n0 * g.C + pl) * (int64_t)HW;
        if (STAGE) {
            __syncthreads();  // the previous plane's reads are done
            const float4 *src = reinterpret_cast<const float4 *>(cb);
            for (int i = threadIdx.x; i < KK * L / 4; i += blockDim.x) reinterpret_cast<float4 *>(slab)[i] = __ldg(src + i);
            __syncthreads();
        }
        const float *sb = STAGE ? slab : cb;
        for (int t = threadIdx.x; t < HW; t += blockDim.x) {
            int iy = t / W, ix = t - iy * W;
            float acc = 0.0f;
            for (int ki = 0; ki < KH; ki++) {
                int oy = iy + g.ph - ki * g.dh;  // divided by the stride below (unit stride: as is)
                if (oy < 0) continue;
                if (g.sh != 1) {
                    if (oy % g.sh) continue;
                    oy /= g.sh;
                }
                if (oy >= OH) continue;
                for (int kj = 0; kj < KW; kj++) {
                    int ox = ix + g.pw - kj * g.dw;
                    if (ox < 0) continue;
                    if (g.sw != 1) {
                        if (ox % g.sw) continue;
                        ox /= g.sw;
                    }
                    if (ox >= OW) continue;
                    acc += STAGE ? sb[(ki * KW + kj) * L + oy * OW + ox] : __ldg(sb + (ki * KW + kj) * L + oy * OW + ox);
                }
            }
            dp[t] = (accum ? dp[t] : 0.0f) + acc;
        }
    }
}

extern "C" void nck_col2im(nck_dev *d, const nck_conv *g, const float *col, float *dx, int64_t n0, int64_t nb,
                           int acc) {
    int64_t total = nb * g->C * g->H * g->W;
    if (total <= 0) return;
    Scope sc(d, "col2im", 0.0, 4.0 * (nb * g->C * g->KH * g->KW * g->OH * g->OW + 2 * total));
    const int64_t slab = g->KH * g->KW * g->OH * g->OW;
    const size_t bytes = (size_t)slab * sizeof(float);
    if (slab % 4 == 0 && ((uintptr_t)col & 15) == 0 && bytes <= 48 * 1024) {
        int64_t planes = nb * g->C, cap = (int64_t)d->sm_count * 8;
        k_col2im<true><<<(int)(planes < cap ? planes : cap), 256, bytes, NCK_STREAM(d)>>>(*g, col, dx, n0, nb, acc);
    } else {
        k_col2im<false><<<plane_grid(d, nb * g->C), 256, 0, NCK_STREAM(d)>>>(*g, col, dx, n0, nb, acc);
    }
    NCK_LAUNCHED(d, 1);
}

// ---- per-channel sums over [N, C, S] (bias gradients) -----------------------------------------------
//
// Block (c, split) sums the planes of channel c for its run of samples with four independent
// accumulators per thread (float4 loads when the plane is 16-byte aligned); the splits are then
// added in order.

template <int V>
__global__ void __launch_bounds__(256) k_chan_sum_partial(const float *__restrict__ x, float *__restrict__ part,
                                                          int64_t N, int64_t C, int64_t S, int64_t per_split,
                                                          float *__restrict__ gb, unsigned *counter) {
    __shared__ float sm[kThreads / 32];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    // four items in flight per thread
    const int64_t pstride = C * S;
    const float *xc = x + (n0 * C + c) * S;
    ChanWalk w;
    w.init((int)(S / V), n1 > n0 ? n1 - n0 : 0);
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    while (w.live()) {
        float v[4][V];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (w.live()) {
                const float *pa = xc + w.na * pstride;
                if constexpr (V == 4) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(pa) + w.ia);
                    v[j][0] = q.x, v[j][1] = q.y, v[j][2] = q.z, v[j][3] = q.w;
                } else {
                    v[j][0] = __ldg(pa + w.ia);
                }
            } else {
#pragma unroll
                for (int k = 0; k < V; k++) v[j][k] = 0.0f;
            }
            w.next();
        }
        if constexpr (V == 4) {
            a0 += v[0][0] + v[0][1], a1 += v[0][2] + v[0][3], a2 += v[1][0] + v[1][1], a3 += v[1][2] + v[1][3];
            a0 += v[2][0] + v[2][1], a1 += v[2][2] + v[2][3], a2 += v[3][0] + v[3][1], a3 += v[3][2] + v[3][3];
        } else {
            a0 += v[0][0], a1 += v[1][0], a2 += v[2][0], a3 += v[3][0];
        }
    }
    float acc = (a0 + a1) + (a2 + a3);
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) s += sm[k];
        part[blockIdx.y * C + c] = s;
    }
    if (last_block_done(counter)) {  // gb[c] += the splits of channel c: 8 lanes per channel, fixed tree
        const unsigned m = 0xFFu << (threadIdx.x & 24);
        for (int64_t cc = threadIdx.x >> 3; cc < C; cc += blockDim.x >> 3) {
            float t = 0.0f;
            for (int k = threadIdx.x & 7; k < (int)gridDim.y; k += 8) t += __ldcg(part + k * C + cc);
            for (int o = 4; o; o >>= 1) t += __shfl_xor_sync(m, t, o, 8);
            if ((threadIdx.x & 7) == 0) gb[cc] += t;
        }
    }
}

extern "C" void nck_conv_bias_grad(nck_dev *d, const float *g, float *gb, int64_t N, int64_t OC, int64_t L) {
    if (N * OC * L <= 0) return;
    Scope sc(d, "conv_bias_grad", 0.0, 4.0 * (N * OC * L + 2 * OC));
    const bool v4 = (L & 3) == 0 && ((uintptr_t)g & 15) == 0;
    static int res4 = 0, res1 = 0;
    if (v4 && !res4) res4 = resident_blocks(d, k_chan_sum_partial<4>, kThreads);
    if (!v4 && !res1) res1 = resident_blocks(d, k_chan_sum_partial<1>, kThreads);
    int64_t splits = (v4 ? res4 : res1) / OC;  // one full wave
    int64_t need = (N * L + ((int64_t)1 << 30) - 1) >> 30; /* a block walks at most 2^30 elements */
    if (splits < need) splits = need;
    if (splits > N) splits = N;
    if (splits < 1) splits = 1;
    int64_t per = (N + splits - 1) / splits;
    splits = (N + per - 1) / per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)OC, (unsigned)splits);
    if (L % 4 == 0 && ((uintptr_t)g & 15) == 0)
        k_chan_sum_partial<4><<<grid, kThreads, 0, NCK_STREAM(d)>>>(g, part, N, OC, L, per, gb, d->counters);
    else
        k_chan_sum_partial<1><<<grid, kThreads, 0, NCK_STREAM(d)>>>(g, part, N, OC, L, per, gb, d->counters);
    NCK_LAUNCHED(d, 1);
}

// ---- direct convolution: each thread reads its receptive field once and produces every output
// channel of its group at that position (Cg * KH * KW <= 32, OCg <= 64) ---------------------------------

// Tap table of one group: for tap k = (c, ki, kj) the input offset c*H*W + ki*dh*W + kj*dw and the
// row / column displacement ki*dh - ph, kj*dw - pw (shared memory, built once per block).
struct Taps {
    int off[32], dy[32], dx[32];
};

__device__ __forceinline__ void build_taps(const nck_conv &g, int CKK, Taps &t) {
    const int KK = (int)(g.KH * g.KW), KW = (int)g.KW, HW = (int)(g.H * g.W);
    for (int k = threadIdx.x; k < CKK; k += blockDim.x) {
        int c = k / KK, kk = k - c * KK, ki = kk / KW, kj = kk - ki * KW;
        t.dy[k] = ki * g.dh - g.ph;
        t.dx[k] = kj * g.dw - g.pw;
        t.off[k] = c * HW + t.dy[k] * (int)g.W + t.dx[k];
    }
}

// receptive field of output position (oy, ox) for the first KT taps (k < CKK live), zero outside
template <int KT>
__device__ __forceinline__ void gather_taps(const float *xg, const Taps &t, int CKK, int oy, int ox, int sh, int sw,
                                            int H, int W, float (&in)[KT]) {
    const int iy0 = oy * sh, ix0 = ox * sw, base = iy0 * W + ix0;
#pragma unroll
    for (int k = 0; k < KT; k++) {
        float v = 0.0f;
        if (k < CKK) {
            int iy = iy0 + t.dy[k], ix = ix0 + t.dx[k];
            if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = __ldg(xg + base + t.off[k]);
        }
        in[k] = v;
    }
}

// y[n, g*OCg + o, l] = bias + sum over taps k in order of w[o, k] * in[k] (fused multiply-adds);
// block (position chunk, group): a grid-stride walk over the flattened (n, l) positions, one output
// position per thread per step; the group's weights and tap table are staged once per block
template <int KT>
__global__ void __launch_bounds__(256) k_conv_direct(nck_conv g, const float *__restrict__ x,
                                                     const float *__restrict__ w, const float *__restrict__ b,
                                                     float *__restrict__ y) {
    __shared__ float ws[64 * 32];
    __shared__ Taps taps;
    const int Cg = (int)(g.C / g.G), OCg = (int)(g.OC / g.G), CKK = Cg * (int)(g.KH * g.KW);
    const int L = (int)(g.OH * g.OW), OW = (int)g.OW, H = (int)g.H, W = (int)g.W;
    const int64_t gi = blockIdx.y;
    for (int i = threadIdx.x; i < OCg * CKK; i += blockDim.x) ws[i] = w[gi * OCg * CKK + i];
    build_taps(g, CKK, taps);
    __syncthreads();
    const int64_t total = g.N * (int64_t)L;
    for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < total; p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = p / L;
        const int l = (int)(p - n * L), oy = l / OW, ox = l - oy * OW;
        const float *xg = x + (n * g.C + gi * Cg) * (int64_t)H * W;
        float *yg = y + (n * g.OC + gi * OCg) * (int64_t)L + l;
        float in[KT];
        gather_taps<KT>(xg, taps, CKK, oy, ox, g.sh, g.sw, H, W, in);
        for (int o = 0; o < OCg; o++) {
            float acc = b ? __ldg(b + gi * OCg + o) : 0.0f;
#pragma unroll
            for (int k = 0; k < KT; k++)
                if (k < CKK) acc = fmaf(ws[o * CKK + k], in[k], acc);
            yg[(int64_t)o * L] = acc;
        }
    }
}

// ---- direct 3x3 convolution of one input channel (stride 1, dilation 1, groups 1): a thread owns one
// output column and four consecutive output rows --------------------------------------------------------

// the 6 x 3 input window of outputs (oy0 .. oy0 + 3, ox): win[kj][i] = x[oy0 - ph + i][ox - pw + kj], zero
// outside the image
__device__ __forceinline__ void window3x4(const float *__restrict__ xn, int H, int W, int ph, int pw, int oy0, int ox,
                                          float (&win)[3][6]) {
#pragma unroll
    for (int i = 0; i < 6; i++) {
        const int iy = oy0 - ph + i;
        const bool rowok = iy >= 0 && iy < H;
#pragma unroll
        for (int kj = 0; kj < 3; kj++) {
            const int ix = ox - pw + kj;
            win[kj][i] = (rowok && ix >= 0 && ix < W) ? __ldg(xn + (int64_t)iy * W + ix) : 0.0f;
        }
    }
}

// y[n, o, oy0 + d, ox] = bias[o] + sum over taps k = (ki, kj) in order of w[o, k] * x (fused multiply-adds,
// the order of the one-position kernel); item = (image, group of 4 rows, column)
__global__ void __launch_bounds__(256) k_conv_direct3(nck_conv g, const float *__restrict__ x,
                                                      const float *__restrict__ w, const float *__restrict__ b,
                                                      float *__restrict__ y, FastDiv dow, FastDiv drg) {
    __shared__ float ws[64 * 9];
    const int OC = (int)g.OC, H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW;
    const uint32_t RG = (uint32_t)(OH + 3) / 4, total = (uint32_t)g.N * RG * (uint32_t)OW;
    for (int i = threadIdx.x; i < OC * 9; i += blockDim.x) ws[i] = w[i];
    __syncthreads();
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = dow.div(t), ox = t - r * (uint32_t)OW, n = drg.div(r), oy0 = 4 * (r - n * RG);
        float win[3][6];
        window3x4(x + (int64_t)n * H * W, H, W, g.ph, g.pw, (int)oy0, (int)ox, win);
        float *yo = y + ((int64_t)n * OC * OH + oy0) * OW + ox;
        const int rows = OH - (int)oy0 < 4 ? OH - (int)oy0 : 4;
        for (int o = 0; o < OC; o++) {
            const float bv = b ? __ldg(b + o) : 0.0f;
            float a[4] = {bv, bv, bv, bv};
#pragma unroll
            for (int ki = 0; ki < 3; ki++)
#pragma unroll
                for (int kj = 0; kj < 3; kj++) {
                    const float wk = ws[o * 9 + ki * 3 + kj];
#pragma unroll
                    for (int d = 0; d < 4; d++) a[d] = fmaf(wk, win[kj][d + ki], a[d]);
                }
            float *yp = yo + (int64_t)o * OH * OW;
#pragma unroll
            for (int d = 0; d < 4; d++)
                if (d < rows) yp[(int64_t)d * OW] = a[d];
        }
    }
}

static bool direct3_ok(const nck_conv *g) {
    return g->G == 1 && g->C == 1 && g->KH == 3 && g->KW == 3 && g->sh == 1 && g->sw == 1 && g->dh == 1 &&
           g->dw == 1 && g->OC <= 64 && g->N * ((g->OH + 3) / 4) * g->OW < ((int64_t)1 << 31);
}

extern "C" void nck_conv_direct_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b,
                                    float *y) {
    int64_t L = g->OH * g->OW, CKK = (g->C / g->G) * g->KH * g->KW;
    if (g->N * g->G * L <= 0) return;
    Scope sc(d, "conv_direct", 2.0 * g->N * g->OC * L * CKK, 4.0 * (g->N * g->C * g->H * g->W + g->N * g->OC * L));
    int64_t bx = (g->N * L + kThreads - 1) / kThreads, cap = ((int64_t)d->sm_count * 8 + g->G - 1) / g->G;
    if (bx > cap) bx = cap;
    if (bx < 1) bx = 1;
    if (direct3_ok(g)) {
        const int64_t items = g->N * ((g->OH + 3) / 4) * g->OW;
        k_conv_direct3<<<grid_for(d, items), kThreads, 0, NCK_STREAM(d)>>>(
            *g, x, w, b, y, make_fastdiv((uint32_t)g->OW), make_fastdiv((uint32_t)((g->OH + 3) / 4)));
        NCK_LAUNCHED(d, 1);
        return;
    }
    dim3 grid((unsigned)bx, (unsigned)g->G);
    if (CKK <= 9) k_conv_direct<9><<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, w, b, y);
    else if (CKK <= 16) k_conv_direct<16><<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, w, b, y);
    else k_conv_direct<32><<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, w, b, y);
    NCK_LAUNCHED(d, 1);
}

// ---- direct weight gradient for few taps per group (Cg * KH * KW <= 32) --------------------------------
//
// dW[g*OCg + o, k] += sum over samples n and positions l of dY[n, g*OCg + o, l] * in_k(n, l). Block
// (split, group * oc-chunk) walks its slice of the flattened (n, l) positions, one per thread, with
// OW_ output channels x KT taps of accumulators in registers; warp shuffles and shared memory reduce
// them to one partial per block, and the splits are added in order by k_direct_dw_combine.
template <int KT, int OCW>
__global__ void __launch_bounds__(128) k_direct_dw_partial(nck_conv g, const float *__restrict__ x,
                                                           const float *__restrict__ gy, float *__restrict__ part,
                                                           int64_t per_split) {
    __shared__ Taps taps;
    __shared__ float red[4][OCW * KT];
    const int Cg = (int)(g.C / g.G), OCg = (int)(g.OC / g.G), CKK = Cg * (int)(g.KH * g.KW);
    const int L = (int)(g.OH * g.OW), OW = (int)g.OW, H = (int)g.H, W = (int)g.W;
    const int chunks = (OCg + OCW - 1) / OCW;
    const int gi = blockIdx.y / chunks, o0 = (blockIdx.y % chunks) * OCW;
    build_taps(g, CKK, taps);
    __syncthreads();
    float acc[OCW][KT];
#pragma unroll
    for (int o = 0; o < OCW; o++)
#pragma unroll
        for (int k = 0; k < KT; k++) acc[o][k] = 0.0f;
    const int64_t total = g.N * (int64_t)L, p0 = blockIdx.x * per_split;
    const int64_t p1 = p0 + per_split < total ? p0 + per_split : total;
    for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        int64_t n = p / L;
        int l = (int)(p - n * L), oy = l / OW, ox = l - oy * OW;
        float in[KT];
        gather_taps<KT>(x + (n * g.C + gi * Cg) * (int64_t)H * W, taps, CKK, oy, ox, g.sh, g.sw, H, W, in);
        const float *gp = gy + (n * g.OC + gi * OCg + o0) * (int64_t)L + l;
#pragma unroll
        for (int o = 0; o < OCW; o++) {
            float gv = (o0 + o < OCg) ? __ldg(gp + (int64_t)o * L) : 0.0f;
#pragma unroll
            for (int k = 0; k < KT; k++) acc[o][k] = fmaf(gv, in[k], acc[o][k]);
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 0; o < OCW; o++)
#pragma unroll
        for (int k = 0; k < KT; k++) {
            float v = acc[o][k];
            for (int s = 16; s; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
            if (lane == 0) red[warp][o * KT + k] = v;
        }
    __syncthreads();
    for (int i = threadIdx.x; i < OCW * KT; i += blockDim.x) {
        int o = i / KT, k = i - o * KT;
        if (o0 + o < OCg && k < CKK) {
            float v = ((red[0][i] + red[1][i]) + red[2][i]) + red[3][i];
            part[((int64_t)blockIdx.x * g.OC + gi * OCg + o0 + o) * CKK + k] = v;
        }
    }
}

// one warp per output: lanes add strided runs of the slices, then a fixed shuffle tree; outputs from n0
// on go to the second array (the bias, when the partials carry it)
__global__ void k_direct_dw_combine(const float *__restrict__ part, int splits, int64_t n, float *__restrict__ gw,
                                    int64_t n0, float *__restrict__ gb) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
        float s = 0.0f;
        for (int k = lane; k < splits; k += 32) s += __ldg(part + k * n + i);
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
            if (i < n0) gw[i] += s;
            else if (gb) gb[i - n0] += s;
        }
    }
}

// The same weight gradient for the 3x3 one-channel case (the forward's fast-path conditions): a
// block takes channels [o0, o0 + 4) and a slice of the (image, group of 4 rows, column) items; per
// item the 6 x 3 window is loaded once and each channel's four dY values feed 36 fused multiply-adds
// into its 9 accumulators. Warp shuffles and shared memory reduce to one partial per block;
// k_direct_dw_combine adds the slices in order.
__global__ void __launch_bounds__(256) k_direct3_dw_partial(nck_conv g, const float *__restrict__ x,
                                                            const float *__restrict__ gy, float *__restrict__ part,
                                                            uint32_t per_split, FastDiv dow, FastDiv drg) {
    constexpr int OCW = 4;
    __shared__ float red[8][OCW * 10];
    const int OC = (int)g.OC, H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW, o0 = blockIdx.y * OCW;
    float acc[OCW][10];  // 9 taps, then the bias (the sum of dY)
#pragma unroll
    for (int o = 0; o < OCW; o++)
#pragma unroll
        for (int k = 0; k < 10; k++) acc[o][k] = 0.0f;
    const uint32_t RG = (uint32_t)(OH + 3) / 4, total = (uint32_t)g.N * RG * (uint32_t)OW, p0 = blockIdx.x * per_split;
    const uint32_t p1 = p0 + per_split < total ? p0 + per_split : total;
    // two items per pass: both items' dY loads (and windows) are issued before either is multiplied,
    // and their products enter the sums in item order (the same order as one item per pass)
    for (uint32_t t0 = p0 + threadIdx.x; t0 < p1; t0 += 2 * blockDim.x) {
        float win[2][3][6], gv[2][OCW][4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint32_t t = t0 + u * blockDim.x;
            if (t >= p1) {
#pragma unroll
                for (int o = 0; o < OCW; o++)
#pragma unroll
                    for (int d = 0; d < 4; d++) gv[u][o][d] = 0.0f;
#pragma unroll
                for (int i = 0; i < 3; i++)
#pragma unroll
                    for (int j = 0; j < 6; j++) win[u][i][j] = 0.0f;
                continue;
            }
            const uint32_t r = dow.div(t), ox = t - r * (uint32_t)OW, n = drg.div(r), oy0 = 4 * (r - n * RG);
            window3x4(x + (int64_t)n * H * W, H, W, g.ph, g.pw, (int)oy0, (int)ox, win[u]);
            const int rows = OH - (int)oy0 < 4 ? OH - (int)oy0 : 4;
            const float *gp = gy + ((int64_t)n * OC * OH + oy0) * OW + ox;
#pragma unroll
            for (int o = 0; o < OCW; o++)
#pragma unroll
                for (int d = 0; d < 4; d++)
                    gv[u][o][d] = (o0 + o < OC && d < rows) ? __ldg(gp + ((int64_t)(o0 + o) * OH + d) * OW) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 2; u++)
#pragma unroll
            for (int o = 0; o < OCW; o++) {
#pragma unroll
                for (int ki = 0; ki < 3; ki++)
#pragma unroll
                    for (int kj = 0; kj < 3; kj++) {
                        float a = acc[o][ki * 3 + kj];
#pragma unroll
                        for (int d = 0; d < 4; d++) a = fmaf(gv[u][o][d], win[u][kj][d + ki], a);
                        acc[o][ki * 3 + kj] = a;
                    }
                acc[o][9] += (gv[u][o][0] + gv[u][o][1]) + (gv[u][o][2] + gv[u][o][3]);
            }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 0; o < OCW; o++)
#pragma unroll
        for (int k = 0; k < 10; k++) {
            float v = acc[o][k];
            for (int sft = 16; sft; sft >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sft);
            if (lane == 0) red[warp][o * 10 + k] = v;
        }
    __syncthreads();
    // partials [block][OC * 9 weights | OC biases]
    for (int i = threadIdx.x; i < OCW * 10; i += blockDim.x) {
        const int o = i / 10, k = i - o * 10;
        if (o0 + o < OC) {
            float v = red[0][i];
            for (int wv = 1; wv < 8; wv++) v += red[wv][i];
            const int64_t row = (int64_t)blockIdx.x * OC * 10;
            part[row + (k < 9 ? (int64_t)(o0 + o) * 9 + k : (int64_t)OC * 9 + o0 + o)] = v;
        }
    }
}

static void direct3_dw_launch(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb) {
    const int64_t chunks = (g->OC + 3) / 4, wsz = g->OC * 10;
    const int64_t total = g->N * ((g->OH + 3) / 4) * g->OW;
    static int resident = 0;  // one full wave of blocks
    if (!resident) resident = resident_blocks(d, k_direct3_dw_partial, kThreads);
    int64_t splits = resident / chunks;
    int64_t maxs = (int64_t)(d->scratch_bytes / sizeof(float)) / wsz;
    if (splits > maxs) splits = maxs;
    if (splits > (total + 255) / 256) splits = (total + 255) / 256;
    if (splits < 1) splits = 1;
    int64_t per = (total + splits - 1) / splits;
    splits = (total + per - 1) / per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)splits, (unsigned)chunks);
    k_direct3_dw_partial<<<grid, kThreads, 0, NCK_STREAM(d)>>>(*g, x, gy, part, (uint32_t)per,
                                                               make_fastdiv((uint32_t)g->OW),
                                                               make_fastdiv((uint32_t)((g->OH + 3) / 4)));
    k_direct_dw_combine<<<grid_for(d, wsz * 32), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, wsz, gw,
                                                                               g->OC * 9, gb);
    NCK_LAUNCHED(d, 2);
}

// Weight (and bias) gradient of a few-tap convolution (groups 1, C*KH*KW + 1 <= 32, OC <= 64) as a
// contraction over positions: a block takes a slice of the (image, position) items in tiles of 64;
// per tile the receptive fields (column k < C*KH*KW, then a column of ones for the bias) and dY of
// every output channel are staged in shared memory, each read from global memory once, and lane k of
// warp w adds dY[p][oc] * col[p][k] for the warp's OCT channels, positions in order. One partial per
// block ([OC][C*KH*KW] weights, then [OC] bias sums); k_direct_dw_combine adds the slices in order.
constexpr int kDwTP = 64;  // positions per tile

template <int OCT>
__global__ void __launch_bounds__(256) k_conv_dw_cols(nck_conv g, const float *__restrict__ x,
                                                      const float *__restrict__ gy, float *__restrict__ part,
                                                      int64_t per_split) {
    __shared__ Taps taps;
    __shared__ float cols[kDwTP][33];
    __shared__ float dys[kDwTP][8 * OCT + 1];
    const int CKK = (int)(g.C * g.KH * g.KW), OC = (int)g.OC;
    const int L = (int)(g.OH * g.OW), OW = (int)g.OW, H = (int)g.H, W = (int)g.W;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, oc0 = warp * OCT;
    build_taps(g, CKK, taps);
    float acc[OCT];
#pragma unroll
    for (int o = 0; o < OCT; o++) acc[o] = 0.0f;
    const int64_t total = g.N * (int64_t)L, p0 = blockIdx.x * per_split;
    const int64_t p1 = p0 + per_split < total ? p0 + per_split : total;
    __syncthreads();
    for (int64_t t0 = p0; t0 < p1; t0 += kDwTP) {
        const int np = (int)(p1 - t0 < kDwTP ? p1 - t0 : kDwTP);
        // receptive fields: thread (q, k-half) gathers half the taps of position q
        for (int e = threadIdx.x; e < kDwTP * 32; e += blockDim.x) {
            const int q = e >> 5, k = e & 31;
            float v = 0.0f;
            if (q < np) {
                const int64_t p = t0 + q, n = p / L;
                const int l = (int)(p - n * L), oy = l / OW, ox = l - oy * OW;
                if (k < CKK) {
                    const int iy = oy * g.sh + taps.dy[k], ix = ox * g.sw + taps.dx[k];
                    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                        v = __ldg(x + n * g.C * (int64_t)H * W + (int64_t)(oy * g.sh) * W + ox * g.sw + taps.off[k]);
                } else if (k == CKK) {
                    v = 1.0f;  // the bias column
                }
            }
            cols[q][k] = v;
        }
        // dY of every channel at the tile's positions (runs of positions are contiguous per channel)
        for (int e = threadIdx.x; e < kDwTP * 8 * OCT; e += blockDim.x) {
            const int oc = e / kDwTP, q = e - oc * kDwTP;
            float v = 0.0f;
            if (q < np && oc < OC) {
                const int64_t p = t0 + q, n = p / L;
                v = __ldg(gy + (n * OC + oc) * (int64_t)L + (p - n * L));
            }
            dys[q][oc] = v;
        }
        __syncthreads();
        for (int q = 0; q < np; q++) {
            const float cv = cols[q][lane];
#pragma unroll
            for (int o = 0; o < OCT; o++) acc[o] = fmaf(dys[q][oc0 + o], cv, acc[o]);
        }
        __syncthreads();
    }
    float *dst = part + (int64_t)blockIdx.x * OC * (CKK + 1);
#pragma unroll
    for (int o = 0; o < OCT; o++) {
        const int oc = oc0 + o;
        if (oc >= OC) continue;
        if (lane < CKK) dst[oc * CKK + lane] = acc[o];
        else if (lane == CKK) dst[OC * CKK + oc] = acc[o];
    }
}

static bool dw_cols_ok(const nck_conv *g) {
    return g->G == 1 && g->C * g->KH * g->KW + 1 <= 32 && g->OC <= 64 && g->N * g->OH * g->OW < ((int64_t)1 << 31);
}

static void dw_cols_launch(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb) {
    const int64_t CKK = g->C * g->KH * g->KW, total = g->N * g->OH * g->OW, wsz = g->OC * (CKK + 1);
    const bool wide = g->OC > 32;
    static int res4 = 0, res8 = 0;
    if (!wide && !res4) res4 = resident_blocks(d, k_conv_dw_cols<4>, 256);
    if (wide && !res8) res8 = resident_blocks(d, k_conv_dw_cols<8>, 256);
    int64_t splits = wide ? res8 : res4;
    const int64_t maxs = (int64_t)(d->scratch_bytes / sizeof(float)) / wsz;
    if (splits > maxs) splits = maxs;
    if (splits > (total + kDwTP - 1) / kDwTP) splits = (total + kDwTP - 1) / kDwTP;
    if (splits < 1) splits = 1;
    int64_t per = (total + splits - 1) / splits;
    per = (per + kDwTP - 1) / kDwTP * kDwTP;
    splits = (total + per - 1) / per;
    float *part = (float *)d->scratch;
    if (wide) k_conv_dw_cols<8><<<(unsigned)splits, 256, 0, NCK_STREAM(d)>>>(*g, x, gy, part, per);
    else k_conv_dw_cols<4><<<(unsigned)splits, 256, 0, NCK_STREAM(d)>>>(*g, x, gy, part, per);
    k_direct_dw_combine<<<grid_for(d, wsz * 32), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, wsz, gw,
                                                                               g->OC * CKK, gb);
    NCK_LAUNCHED(d, 2);
}

template <int KT, int OCW>
static void direct_dw_launch(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw) {
    const int64_t OCg = g->OC / g->G, CKK = (g->C / g->G) * g->KH * g->KW, L = g->OH * g->OW;
    const int64_t chunks = (OCg + OCW - 1) / OCW, total = g->N * L, wsz = g->OC * CKK;
    static int resident = 0;  // one full wave of blocks
    if (!resident) resident = resident_blocks(d, k_direct_dw_partial<KT, OCW>, 128);
    int64_t splits = resident / (g->G * chunks);
    int64_t maxs = (int64_t)(d->scratch_bytes / sizeof(float)) / wsz;
    if (splits > maxs) splits = maxs;
    if (splits > (total + 127) / 128) splits = (total + 127) / 128;
    if (splits < 1) splits = 1;
    int64_t per = (total + splits - 1) / splits;
    splits = (total + per - 1) / per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)splits, (unsigned)(g->G * chunks));
    k_direct_dw_partial<KT, OCW><<<grid, 128, 0, NCK_STREAM(d)>>>(*g, x, gy, part, per);
    k_direct_dw_combine<<<grid_for(d, wsz * 32), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, wsz, gw, wsz,
                                                                               nullptr);
    NCK_LAUNCHED(d, 2);
}

extern "C" int nck_conv_direct3_ok(const nck_conv *g) { return direct3_ok(g); }

extern "C" int nck_conv_direct_dw_bias_ok(const nck_conv *g) { return direct3_ok(g) || dw_cols_ok(g); }

extern "C" int nck_conv_direct_dw(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw,
                                  float *gb) {
    int64_t CKK = (g->C / g->G) * g->KH * g->KW, L = g->OH * g->OW;
    if (g->N * L <= 0 || CKK <= 0) return 0;
    Scope sc(d, "conv_direct_dw", 2.0 * g->N * g->OC * L * CKK,
             4.0 * (g->N * g->C * g->H * g->W + g->N * g->OC * L + 2 * g->OC * CKK));
    if (direct3_ok(g)) {
        direct3_dw_launch(d, g, x, gy, gw, gb);
        return gb != nullptr;
    }
    if (dw_cols_ok(g)) {
        dw_cols_launch(d, g, x, gy, gw, gb);
        return gb != nullptr;
    }
    if (CKK <= 9) direct_dw_launch<9, 8>(d, g, x, gy, gw);
    else if (CKK <= 16) direct_dw_launch<16, 4>(d, g, x, gy, gw);
    else direct_dw_launch<32, 2>(d, g, x, gy, gw);
    return 0;
}

// ---- depthwise (groups == C == OC) ---------------------------------------------------------------
//
// One block works on a tile of consecutive rows (full width) of one (sample, channel) plane. The
// input rows the tile needs, padding included, are staged in shared memory with coalesced row loads;
// the out-of-image padding is stored as zeros, so the tap loops need no bounds tests (a zero term
// leaves a sum unchanged). Sums run in newch's order (engine/src/ops/ops_conv.c dw_fwd_range :192,
// dw_dx_range :222): the forward starts from the bias and adds taps (ki, kj) row-major; the input
// gradient adds, for each element, its taps in the order newch's row passes reach it (ki from the
// last kernel row up, kj ascending). With unit column stride newch adds through its fused
// multiply-add axpy, otherwise with a product and a sum; the kernels do the same, so both are
// bit-identical to newch's AVX2 tier.

namespace {

constexpr int kDwThreads = 256;
constexpr int kDwTileOut = 2048; // outputs per block (8 per thread)

struct DwPlan {
    int rows;     // output rows per tile (input-gradient rows for dx)
    int tiles;    // tiles per plane
    int srows;    // staged rows
    int scols;    // staged row width
};

// Stages rows [r0, r0 + nr) x columns [c0, c0 + SW) of a plane (H x W) in shared memory, zero outside.
__device__ __forceinline__ void dw_stage(const float *__restrict__ src, int H, int W, int r0, int nr, int c0, int SW,
                                         float *__restrict__ sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int r = warp; r < nr; r += nw) {
        const int iy = r0 + r;
        const bool row_ok = iy >= 0 && iy < H;
        const float *row = src + (int64_t)iy * W;
        for (int cc = lane; cc < SW; cc += 32) {
            const int ix = c0 + cc;
            sm[r * SW + cc] = (row_ok && ix >= 0 && ix < W) ? __ldg(row + ix) : 0.0f;
        }
    }
}

// KH_T, KW_T: the kernel size when fixed at compile time (3 x 3), 0 for any size
template <bool FMA, int KH_T, int KW_T>
__global__ void __launch_bounds__(kDwThreads) k_dw_fwd(nck_conv g, const float *__restrict__ x,
                                                       const float *__restrict__ w, const float *__restrict__ b,
                                                       float *__restrict__ y, DwPlan pl, FastDiv div_ow) {
    extern __shared__ float sm[];
    float *wk = sm;              // the channel's taps
    float *sx = sm + NCK_DW_MAX_TAPS;
    const int64_t plane = blockIdx.x / pl.tiles;
    const int tile = (int)(blockIdx.x - plane * pl.tiles);
    const int c = (int)(plane % g.C);
    const int H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW;
    const int KH = KH_T ? KH_T : (int)g.KH, KW = KW_T ? KW_T : (int)g.KW;
    const int oy0 = tile * pl.rows, oy1 = min(OH, oy0 + pl.rows);
    const int KK = KH * KW;
    if (threadIdx.x < KK) wk[threadIdx.x] = __ldg(w + (int64_t)c * KK + threadIdx.x);
    dw_stage(x + plane * (int64_t)H * W, H, W, oy0 * g.sh - g.ph, pl.srows, -g.pw, pl.scols, sx);
    __syncthreads();
    const float bias = b ? __ldg(b + c) : 0.0f;
    float *yp = y + plane * (int64_t)OH * OW + (int64_t)oy0 * OW;
    const int n = (oy1 - oy0) * OW;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int oy = (int)div_ow.div((uint32_t)t), ox = t - oy * OW;
        const float *base = sx + oy * g.sh * pl.scols + ox * g.sw;
        float acc = bias;
#pragma unroll
        for (int ki = 0; ki < KH; ki++) {
            const float *rowp = base + ki * g.dh * pl.scols;
#pragma unroll
            for (int kj = 0; kj < KW; kj++) {
                const float wv = wk[ki * KW + kj], xv = rowp[kj * g.dw];
                acc = FMA ? fmaf(wv, xv, acc) : acc + wv * xv;
            }
        }
        yp[t] = acc;
    }
}

// dx rows [iy0, iy1) of a plane; the gy rows they draw on are staged (zero outside the output).
template <bool FMA, bool UNIT, int KH_T, int KW_T>
__global__ void __launch_bounds__(kDwThreads) k_dw_dx(nck_conv g, const float *__restrict__ gy,
                                                      const float *__restrict__ w, float *__restrict__ gx, int acc_in,
                                                      DwPlan pl, FastDiv div_w) {
    extern __shared__ float sm[];
    float *wk = sm;
    float *sg = sm + NCK_DW_MAX_TAPS;
    const int64_t plane = blockIdx.x / pl.tiles;
    const int tile = (int)(blockIdx.x - plane * pl.tiles);
    const int c = (int)(plane % g.C);
    const int H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW;
    const int KH = KH_T ? KH_T : (int)g.KH, KW = KW_T ? KW_T : (int)g.KW;
    const int iy0 = tile * pl.rows, iy1 = min(H, iy0 + pl.rows);
    const int KK = KH * KW;
    if (threadIdx.x < KK) wk[threadIdx.x] = __ldg(w + (int64_t)c * KK + threadIdx.x);
    // output rows that reach this tile: oy in [oy_lo, oy_lo + srows), staged from column -cpad
    const int span = (KH - 1) * g.dh;
    const int oy_lo = UNIT ? iy0 + g.ph - span : (iy0 + g.ph - span >= 0 ? (iy0 + g.ph - span) / g.sh : -((g.sh - 1 - (iy0 + g.ph - span)) / g.sh));
    const int cpad = UNIT ? (KW - 1) * g.dw - g.pw : 0;
    dw_stage(gy + plane * (int64_t)OH * OW, OH, OW, oy_lo, pl.srows, -cpad, pl.scols, sg);
    __syncthreads();
    float *xp = gx + plane * (int64_t)H * W + (int64_t)iy0 * W;
    const int n = (iy1 - iy0) * W;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int r = (int)div_w.div((uint32_t)t), ix = t - r * W, iy = iy0 + r;
        float acc = acc_in ? xp[t] : 0.0f;
#pragma unroll
        for (int ki = KH - 1; ki >= 0; ki--) {
            const int ty = iy + g.ph - ki * g.dh;
            int oy;
            if (UNIT) {
                oy = ty;
            } else {
                if (ty < 0 || ty % g.sh) continue;
                oy = ty / g.sh;
                if (oy >= OH) continue;
            }
            const float *rowp = sg + (oy - oy_lo) * pl.scols;
#pragma unroll
            for (int kj = 0; kj < KW; kj++) {
                const int tx = ix + g.pw - kj * g.dw;
                float gv;
                if (UNIT) {
                    gv = rowp[tx + cpad];
                } else {
                    if (tx < 0 || tx % g.sw) continue;
                    const int ox = tx / g.sw;
                    if (ox >= OW) continue;
                    gv = rowp[ox];
                }
                const float wv = wk[ki * KW + kj];
                acc = FMA ? fmaf(wv, gv, acc) : acc + wv * gv;
            }
        }
        xp[t] = acc;
    }
}

// Weight and bias gradients: block (c, split) walks the (plane, row tile) items of its samples; a
// thread keeps one running sum per tap (and one for the bias) over its output positions; the block
// then adds the threads' sums in a fixed tree, and a combine kernel adds the splits in order.
template <int KH_T, int KW_T>
__global__ void __launch_bounds__(kDwThreads) k_dw_dw_partial(nck_conv g, const float *__restrict__ x,
                                                              const float *__restrict__ gy, float *__restrict__ part,
                                                              int64_t per_split, DwPlan pl, FastDiv div_ow) {
    extern __shared__ float sm[];
    __shared__ float red[kDwThreads / 32][NCK_DW_MAX_TAPS + 1];
    const int c = blockIdx.x;
    const int64_t n0 = blockIdx.y * per_split, n1 = min(g.N, n0 + per_split);
    const int H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW;
    const int KH = KH_T ? KH_T : (int)g.KH, KW = KW_T ? KW_T : (int)g.KW;
    const int KK = KH * KW;
    constexpr int NA = (KH_T && KW_T) ? KH_T * KW_T : NCK_DW_MAX_TAPS; // tap sums; the bias sum is separate
    float acc[NA];
    float bsum = 0.0f;
#pragma unroll
    for (int k = 0; k < NA; k++) acc[k] = 0.0f;
    for (int64_t nn = n0; nn < n1; nn++) {
        const int64_t plane = nn * g.C + c;
        const float *xp = x + plane * (int64_t)H * W, *gp = gy + plane * (int64_t)OH * OW;
        for (int tile = 0; tile < pl.tiles; tile++) {
            const int oy0 = tile * pl.rows, oy1 = min(OH, oy0 + pl.rows);
            __syncthreads(); // the previous item's readers are done with the staged rows
            dw_stage(xp, H, W, oy0 * g.sh - g.ph, pl.srows, -g.pw, pl.scols, sm);
            __syncthreads();
            const int n = (oy1 - oy0) * OW;
            const float *gt = gp + (int64_t)oy0 * OW;
            for (int t = threadIdx.x; t < n; t += blockDim.x) {
                const int oy = (int)div_ow.div((uint32_t)t), ox = t - oy * OW;
                const float gv = __ldg(gt + t);
                const float *base = sm + oy * g.sh * pl.scols + ox * g.sw;
#pragma unroll
                for (int ki = 0; ki < KH; ki++)
#pragma unroll
                    for (int kj = 0; kj < KW; kj++) {
                        const int k = ki * KW + kj;
                        acc[k] = fmaf(base[ki * g.dh * pl.scols + kj * g.dw], gv, acc[k]);
                    }
                bsum += gv;
            }
        }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k <= NA; k++) {
        if (k < NA && k >= KK) continue;
        float v = k < NA ? acc[k] : bsum;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[wid][k < NA ? k : NCK_DW_MAX_TAPS] = v;
    }
    __syncthreads();
    if (threadIdx.x <= NCK_DW_MAX_TAPS && (threadIdx.x < KK || threadIdx.x == NCK_DW_MAX_TAPS)) {
        float s = 0.0f;
        for (int q = 0; q < (int)(blockDim.x >> 5); q++) s += red[q][threadIdx.x];
        part[((int64_t)blockIdx.y * g.C + c) * (NCK_DW_MAX_TAPS + 1) + threadIdx.x] = s;
    }
}

__global__ void k_dw_dw_combine(const float *__restrict__ part, int splits, int64_t C, int KK, float *__restrict__ gw,
                                float *__restrict__ gb) {
    const int64_t per = NCK_DW_MAX_TAPS + 1, total = C * (KK + 1);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = t / (KK + 1);
        const int k = (int)(t - c * (KK + 1));
        const int slot = k < KK ? k : NCK_DW_MAX_TAPS;
        if (k == KK && !gb) continue;
        float s = 0.0f;
        for (int q = 0; q < splits; q++) s += part[(q * C + c) * per + slot];
        if (k < KK) gw[c * KK + k] += s;
        else gb[c] += s;
    }
}

// ---- 3 x 3, stride 1, dilation 1, output rows a multiple of 4 wide: strips of four outputs -------
// A thread takes four consecutive outputs of a row: the 3 x 6 input window they share is read once
// (L1-cached loads, zero outside the image) instead of staged behind block barriers, and the four
// outputs keep the per-element arithmetic of the tiled kernels above (forward: the bias, then the taps
// row-major; input gradient: kernel rows from the last up, columns ascending), so results are the
// same bit for bit. The weight gradient keeps one running sum per tap over the thread's strips, plane
// by plane, its four outputs in column order.

struct Strip3 {
    uint32_t planes, OH, OW4;  // strips: planes * OH * OW4
    FastDiv dow4, doh;
};

__device__ __forceinline__ void strip_pos(const Strip3 &g, uint32_t t, uint32_t &plane, int &oy, int &ox) {
    const uint32_t r = g.dow4.div(t), q = t - r * g.OW4;
    plane = g.doh.div(r);
    oy = (int)(r - plane * g.OH), ox = (int)(4 * q);
}

// rows r0 .. r0 + 2, columns c0 .. c0 + 5 of a plane (H x W), zero outside
__device__ __forceinline__ void window36(const float *__restrict__ p, int H, int W, int r0, int c0, float (&v)[3][6]) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int y = r0 + i;
        const bool rok = y >= 0 && y < H;
#pragma unroll
        for (int j = 0; j < 6; j++) {
            const int x = c0 + j;
            v[i][j] = rok && x >= 0 && x < W ? __ldg(p + (int64_t)y * W + x) : 0.0f;
        }
    }
}

// window36 when columns c0 + 1 .. c0 + 4 are one aligned float4 (c0 + 1 a multiple of 4, W a multiple of
// 4, p 16-byte aligned: a padding of 1 with strips of four): three loads per row instead of six
__device__ __forceinline__ void window36v(const float *__restrict__ p, int H, int W, int r0, int c0,
                                          float (&v)[3][6]) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int y = r0 + i;
        const bool rok = y >= 0 && y < H;
        const float *row = p + (int64_t)(rok ? y : 0) * W;
        const float4 m = rok ? __ldg(reinterpret_cast<const float4 *>(row + c0 + 1)) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i][0] = rok && c0 >= 0 ? __ldg(row + c0) : 0.0f;
        v[i][1] = m.x, v[i][2] = m.y, v[i][3] = m.z, v[i][4] = m.w;
        v[i][5] = rok && c0 + 5 < W ? __ldg(row + c0 + 5) : 0.0f;
    }
}

__global__ void __launch_bounds__(256) k_dw3_fwd(nck_conv g, Strip3 st, const float *__restrict__ x,
                                                 const float *__restrict__ w, const float *__restrict__ b,
                                                 float *__restrict__ y) {
    const uint32_t total = st.planes * st.OH * st.OW4;
    const int H = (int)g.H, W = (int)g.W, OW = (int)g.OW;
    const bool vec = g.ph == 1 && g.pw == 1 && (W & 3) == 0 && ((uintptr_t)x & 15) == 0;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        uint32_t plane;
        int oy, ox;
        strip_pos(st, t, plane, oy, ox);
        const int c = (int)(plane % (uint32_t)g.C);
        float wk[9];
#pragma unroll
        for (int k = 0; k < 9; k++) wk[k] = __ldg(w + c * 9 + k);
        float v[3][6];
        if (vec) window36v(x + (int64_t)plane * H * W, H, W, oy - 1, ox - 1, v);
        else window36(x + (int64_t)plane * H * W, H, W, oy - g.ph, ox - g.pw, v);
        const float bias = b ? __ldg(b + c) : 0.0f;
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float acc = bias;
#pragma unroll
            for (int ki = 0; ki < 3; ki++)
#pragma unroll
                for (int kj = 0; kj < 3; kj++) acc = fmaf(wk[ki * 3 + kj], v[ki][e + kj], acc);
            o[e] = acc;
        }
        *reinterpret_cast<float4 *>(y + (int64_t)plane * g.OH * OW + (int64_t)oy * OW + ox) =
            make_float4(o[0], o[1], o[2], o[3]);
    }
}

// input gradient: strips of the input plane (H x W, W a multiple of 4); gy rows iy + ph - ki
__global__ void __launch_bounds__(256) k_dw3_dx(nck_conv g, Strip3 st, const float *__restrict__ gy,
                                                const float *__restrict__ w, float *__restrict__ gx, int acc_in) {
    const uint32_t total = st.planes * st.OH * st.OW4;
    const int H = (int)g.H, W = (int)g.W, OH = (int)g.OH, OW = (int)g.OW;
    const bool vec = g.ph == 1 && g.pw == 1 && (OW & 3) == 0 && ((uintptr_t)gy & 15) == 0;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        uint32_t plane;
        int iy, ix;
        strip_pos(st, t, plane, iy, ix);
        const int c = (int)(plane % (uint32_t)g.C);
        float wk[9];
#pragma unroll
        for (int k = 0; k < 9; k++) wk[k] = __ldg(w + c * 9 + k);
        // v[i][j] = gy[iy + ph - 2 + i][ix + pw - 2 + j]: tap (ki, kj) of output e reads v[2 - ki][e + 2 - kj]
        float v[3][6];
        if (vec) window36v(gy + (int64_t)plane * OH * OW, OH, OW, iy - 1, ix - 1, v);
        else window36(gy + (int64_t)plane * OH * OW, OH, OW, iy + g.ph - 2, ix + g.pw - 2, v);
        float *dst = gx + (int64_t)plane * H * W + (int64_t)iy * W + ix;
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (acc_in) {
            const float4 a = *reinterpret_cast<const float4 *>(dst);
            o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float acc = o[e];
#pragma unroll
            for (int ki = 2; ki >= 0; ki--)
#pragma unroll
                for (int kj = 0; kj < 3; kj++) acc = fmaf(wk[ki * 3 + kj], v[2 - ki][e + 2 - kj], acc);
            o[e] = acc;
        }
        *reinterpret_cast<float4 *>(dst) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// weight and bias gradient partials: block (c, split) over the planes of its samples
__global__ void __launch_bounds__(256) k_dw3_dw_partial(nck_conv g, Strip3 st, const float *__restrict__ x,
                                                        const float *__restrict__ gy, float *__restrict__ part,
                                                        int64_t per_split) {
    __shared__ float red[8][NCK_DW_MAX_TAPS + 1];
    const int c = blockIdx.x;
    const int64_t n0 = blockIdx.y * per_split, n1 = min(g.N, n0 + per_split);
    const int H = (int)g.H, W = (int)g.W, OW = (int)g.OW;
    const bool vec = g.ph == 1 && g.pw == 1 && (W & 3) == 0 && ((uintptr_t)x & 15) == 0;
    const uint32_t strips = st.OH * st.OW4;
    float acc[9], bsum = 0.0f;
#pragma unroll
    for (int k = 0; k < 9; k++) acc[k] = 0.0f;
    for (int64_t nn = n0; nn < n1; nn++) {
        const int64_t plane = nn * g.C + c;
        const float *xp = x + plane * H * W, *gp = gy + plane * (int64_t)g.OH * OW;
        for (uint32_t q = threadIdx.x; q < strips; q += blockDim.x) {
            const uint32_t oy = st.dow4.div(q);
            const int ox = (int)(4 * (q - oy * st.OW4));
            const float4 g4 = __ldg(reinterpret_cast<const float4 *>(gp + (int64_t)oy * OW + ox));
            float v[3][6];
            if (vec) window36v(xp, H, W, (int)oy - 1, ox - 1, v);
            else window36(xp, H, W, (int)oy - g.ph, ox - g.pw, v);
            const float ge[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
#pragma unroll
                for (int ki = 0; ki < 3; ki++)
#pragma unroll
                    for (int kj = 0; kj < 3; kj++) acc[ki * 3 + kj] = fmaf(v[ki][e + kj], ge[e], acc[ki * 3 + kj]);
                bsum += ge[e];
            }
        }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k <= 9; k++) {
        float v = k < 9 ? acc[k] : bsum;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[wid][k < 9 ? k : NCK_DW_MAX_TAPS] = v;
    }
    __syncthreads();
    if (threadIdx.x < 9 || threadIdx.x == NCK_DW_MAX_TAPS) {
        float s = 0.0f;
        for (int q = 0; q < (int)(blockDim.x >> 5); q++) s += red[q][threadIdx.x];
        part[((int64_t)blockIdx.y * g.C + c) * (NCK_DW_MAX_TAPS + 1) + threadIdx.x] = s;
    }
}

bool dw3_ok(const nck_conv *g, int64_t rows, int64_t cols) {
    return g->KH == 3 && g->KW == 3 && g->sh == 1 && g->sw == 1 && g->dh == 1 && g->dw == 1 && cols % 4 == 0 &&
           g->N * g->C * rows * cols < ((int64_t)1 << 31) && g->ph <= 2 && g->pw <= 2;
}

Strip3 strip3(int64_t planes, int64_t rows, int64_t cols) {
    Strip3 s;
    s.planes = (uint32_t)planes, s.OH = (uint32_t)rows, s.OW4 = (uint32_t)(cols / 4);
    s.dow4 = make_fastdiv(s.OW4), s.doh = make_fastdiv(s.OH);
    return s;
}

// rows per tile so that a tile has about kDwTileOut outputs; staged rows and width for it
DwPlan dw_plan_out(const nck_conv *g) {
    DwPlan p;
    const int64_t OW = g->OW > 0 ? g->OW : 1;
    int rows = (int)(kDwTileOut / OW);
    if (rows < 1) rows = 1;
    if (rows > g->OH) rows = (int)g->OH;
    p.rows = rows > 0 ? rows : 1;
    p.tiles = (int)((g->OH + p.rows - 1) / p.rows);
    p.srows = (p.rows - 1) * g->sh + (int)(g->KH - 1) * g->dh + 1;
    p.scols = (int)((g->OW - 1) * g->sw + (g->KW - 1) * g->dw + 1);
    return p;
}

size_t dw_smem(const DwPlan &p) { return sizeof(float) * ((size_t)NCK_DW_MAX_TAPS + (size_t)p.srows * p.scols); }

} // namespace

// Plans whose staged rows fit in shared memory take the tiled kernels (every practical depthwise
// layer: a 3x3 over a 4096-wide row needs ~50 KB).
static bool dw_fits(const DwPlan &p) { return dw_smem(p) <= (size_t)200 * 1024; }

extern "C" int nck_dw_ok(const nck_conv *g) {
    if (g->KH * g->KW > NCK_DW_MAX_TAPS || g->H * g->W >= ((int64_t)1 << 31) || g->OH * g->OW >= ((int64_t)1 << 31))
        return 0;
    DwPlan a = dw_plan_out(g);
    nck_conv t = *g;
    t.OH = g->H, t.OW = g->W; /* the input-gradient tiling, sized on the input plane */
    DwPlan b = dw_plan_out(&t);
    b.srows = (b.rows - 1 + (int)(g->KH - 1) * g->dh) / g->sh + 2;
    b.scols = (int)(g->sh == 1 && g->sw == 1 ? g->W + (g->KW - 1) * g->dw : g->OW);
    return dw_fits(a) && dw_fits(b);
}

extern "C" void nck_dw_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b, float *y) {
    const int64_t total = g->N * g->C * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, "dw_fwd", 2.0 * total * g->KH * g->KW, 4.0 * (g->N * g->C * g->H * g->W + total));
    if (dw3_ok(g, g->OH, g->OW) && (((uintptr_t)x | (uintptr_t)y) & 15) == 0) {
        const Strip3 st = strip3(g->N * g->C, g->OH, g->OW);
        k_dw3_fwd<<<grid_for(d, total / 4), 256, 0, NCK_STREAM(d)>>>(*g, st, x, w, b, y);
        NCK_LAUNCHED(d, 1);
        return;
    }
    const DwPlan pl = dw_plan_out(g);
    const size_t smem = dw_smem(pl);
    const int64_t blocks = g->N * g->C * pl.tiles;
    const bool k3 = g->KH == 3 && g->KW == 3;
    auto k = g->sw == 1 ? (k3 ? k_dw_fwd<true, 3, 3> : k_dw_fwd<true, 0, 0>)
                        : (k3 ? k_dw_fwd<false, 3, 3> : k_dw_fwd<false, 0, 0>);
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)blocks, kDwThreads, smem, NCK_STREAM(d)>>>(*g, x, w, b, y, pl, make_fastdiv((uint32_t)g->OW));
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_dw_dx(nck_dev *d, const nck_conv *g, const float *gy, const float *w, float *gx, int acc) {
    const int64_t total = g->N * g->C * g->H * g->W;
    if (total <= 0) return;
    Scope sc(d, "dw_dx", 2.0 * g->N * g->C * g->OH * g->OW * g->KH * g->KW,
             4.0 * (g->N * g->C * g->OH * g->OW + (acc ? 2 : 1) * total));
    if (dw3_ok(g, g->H, g->W) && (((uintptr_t)gy | (uintptr_t)gx) & 15) == 0) {
        const Strip3 st = strip3(g->N * g->C, g->H, g->W);
        k_dw3_dx<<<grid_for(d, total / 4), 256, 0, NCK_STREAM(d)>>>(*g, st, gy, w, gx, acc);
        NCK_LAUNCHED(d, 1);
        return;
    }
    nck_conv t = *g;
    t.OH = g->H, t.OW = g->W;
    DwPlan pl = dw_plan_out(&t); /* rows of the input plane per tile */
    const bool unit = g->sh == 1 && g->sw == 1;
    /* staged gy rows: those reached from the tile's rows, plus one for the rounding of the first */
    pl.srows = unit ? pl.rows + (int)(g->KH - 1) * g->dh : (pl.rows - 1 + (int)(g->KH - 1) * g->dh) / g->sh + 2;
    pl.scols = (int)(unit ? g->W + (g->KW - 1) * g->dw : g->OW);
    const size_t smem = dw_smem(pl);
    const int64_t blocks = g->N * g->C * pl.tiles;
    const bool k3 = g->KH == 3 && g->KW == 3;
    /* unit strides: newch's axpy rows (fused multiply-adds) */
    auto k = unit ? (k3 ? k_dw_dx<true, true, 3, 3> : k_dw_dx<true, true, 0, 0>)
                  : (g->sw == 1 ? (k3 ? k_dw_dx<true, false, 3, 3> : k_dw_dx<true, false, 0, 0>)
                                : (k3 ? k_dw_dx<false, false, 3, 3> : k_dw_dx<false, false, 0, 0>));
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)blocks, kDwThreads, smem, NCK_STREAM(d)>>>(*g, gy, w, gx, acc, pl, make_fastdiv((uint32_t)g->W));
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_dw_dw(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb) {
    const int KK = (int)(g->KH * g->KW);
    if (g->N * g->C <= 0 || KK <= 0 || KK > NCK_DW_MAX_TAPS) return;
    Scope sc(d, "dw_dw", 2.0 * g->N * g->C * g->OH * g->OW * KK,
             4.0 * (g->N * g->C * (g->H * g->W + g->OH * g->OW)));
    float *part = (float *)d->scratch;
    if (dw3_ok(g, g->OH, g->OW) && ((uintptr_t)gy & 15) == 0) {
        static int res = 0;
        if (!res) res = resident_blocks(d, k_dw3_dw_partial, 256);
        int64_t splits = (res + g->C - 1) / g->C;
        if (splits > g->N) splits = g->N;
        if (splits < 1) splits = 1;
        const int64_t per = (g->N + splits - 1) / splits;
        splits = (g->N + per - 1) / per;
        const Strip3 st = strip3(1, g->OH, g->OW);
        dim3 grid((unsigned)g->C, (unsigned)splits);
        k_dw3_dw_partial<<<grid, 256, 0, NCK_STREAM(d)>>>(*g, st, x, gy, part, per);
        k_dw_dw_combine<<<grid_for(d, g->C * (KK + 1)), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, g->C, KK, gw,
                                                                                     gb);
        NCK_LAUNCHED(d, 2);
        return;
    }
    const DwPlan pl = dw_plan_out(g);
    const size_t smem = sizeof(float) * (size_t)pl.srows * pl.scols;
    const bool k3 = g->KH == 3 && g->KW == 3;
    auto kp = k3 ? k_dw_dw_partial<3, 3> : k_dw_dw_partial<0, 0>;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kp, kDwThreads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 2;
    cudaGetLastError();
    int64_t splits = ((int64_t)d->sm_count * per_sm + g->C - 1) / g->C;
    if (splits > g->N) splits = g->N;
    if (splits < 1) splits = 1;
    const int64_t per = (g->N + splits - 1) / splits;
    splits = (g->N + per - 1) / per;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)g->C, (unsigned)splits);
    kp<<<grid, kDwThreads, smem, NCK_STREAM(d)>>>(*g, x, gy, part, per, pl, make_fastdiv((uint32_t)g->OW));
    k_dw_dw_combine<<<grid_for(d, g->C * (KK + 1)), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, g->C, KK, gw, gb);
    NCK_LAUNCHED(d, 2);
}

// ---- pooling ---------------------------------------------------------------------------------------------

// Pooling kernels index with I = uint32_t when every index fits (the common case: integer division
// is several times cheaper than with 64-bit operands), else int64_t.
template <typename I>
__global__ void k_pool_fwd(nck_conv g, const float *__restrict__ x, float *__restrict__ y, int32_t *__restrict__ arg,
                           int is_max, FastDiv divOW, FastDiv divOH) {
    const I OW = (I)g.OW, OH = (I)g.OH, H = (I)g.H, W = (I)g.W, KH = (I)g.KH, KW = (I)g.KW;
    const I total = (I)(g.N * g.C) * OH * OW;
    const float inv = 1.0f / (float)(g.KH * g.KW);
    for (I t = blockIdx.x * (I)blockDim.x + threadIdx.x; t < total; t += (I)gridDim.x * blockDim.x) {
        I r, plane;
        if constexpr (sizeof(I) == 4) r = divOW.div(t), plane = divOH.div(r);
        else r = t / OW, plane = r / OH;
        I ox = t - r * OW, oy = r - plane * OH;
        const float *xp = x + (int64_t)plane * H * W;
        float best = -INFINITY, acc = 0.0f;
        int32_t bi = -1;
        const int64_t iy0 = (int64_t)oy * g.sh - g.ph, ix0 = (int64_t)ox * g.sw - g.pw;
        for (I ki = 0; ki < KH; ki++) {
            int64_t iy = iy0 + (int64_t)ki;
            if (iy < 0 || iy >= (int64_t)H) continue;
            for (I kj = 0; kj < KW; kj++) {
                int64_t ix = ix0 + (int64_t)kj;
                if (ix < 0 || ix >= (int64_t)W) continue;
                float v = __ldg(xp + iy * (int64_t)W + ix);
                acc += v;
                if (v > best || bi < 0) best = v, bi = (int32_t)(iy * (int64_t)W + ix);
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

static bool small_index(int64_t n) { return n > 0 && n < ((int64_t)1 << 31); }

// 2x2 max pooling with stride 2 and no padding, input width a multiple of 4: a thread reads one float4
// from each of the two input rows of a window pair and writes two adjacent outputs (taps in newch's
// order, the first maximum kept)
__device__ __forceinline__ void max4(float a, float b, float c, float d, int32_t ia, int32_t W, float &best,
                                     int32_t &bi) {
    best = a, bi = ia;
    if (b > best) best = b, bi = ia + 1;
    if (c > best) best = c, bi = ia + W;
    if (d > best) best = d, bi = ia + W + 1;
}

__global__ void __launch_bounds__(256) k_maxpool2x2(const float *__restrict__ x, float *__restrict__ y,
                                                    int32_t *__restrict__ arg, uint32_t planes, uint32_t H, uint32_t W,
                                                    uint32_t OH, uint32_t OW) {
    const uint32_t pairs = (OW + 1) / 2, total = planes * OH * pairs;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = t / pairs, q = t - r * pairs, pl = r / OH, oy = r - pl * OH;
        const float *r0 = x + (size_t)pl * H * W + (size_t)(2 * oy) * W;
        const float4 a = __ldg(reinterpret_cast<const float4 *>(r0) + q);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(r0 + W) + q);
        const int32_t i0 = (int32_t)(2 * oy * W + 4 * q);
        const size_t o = (size_t)pl * OH * OW + (size_t)oy * OW + 2 * q;
        float best;
        int32_t bi;
        max4(a.x, a.y, b.x, b.y, i0, (int32_t)W, best, bi);
        y[o] = best;
        arg[o] = bi;
        if (2 * q + 1 < OW) {
            max4(a.z, a.w, b.z, b.w, i0 + 2, (int32_t)W, best, bi);
            y[o + 1] = best;
            arg[o + 1] = bi;
        }
    }
}

// the same for an even input width: one output per thread from one float2 of each window row
__global__ void __launch_bounds__(256) k_maxpool2x2_w2(const float *__restrict__ x, float *__restrict__ y,
                                                       int32_t *__restrict__ arg, uint32_t planes, uint32_t H,
                                                       uint32_t W, uint32_t OH, uint32_t OW, FastDiv dow, FastDiv doh) {
    const uint32_t total = planes * OH * OW;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = dow.div(t), ox = t - r * OW, pl = doh.div(r), oy = r - pl * OH;
        const float *r0 = x + (size_t)pl * H * W + (size_t)(2 * oy) * W + 2 * ox;
        const float2 a = __ldg(reinterpret_cast<const float2 *>(r0));
        const float2 b = __ldg(reinterpret_cast<const float2 *>(r0 + W));
        float best;
        int32_t bi;
        max4(a.x, a.y, b.x, b.y, (int32_t)(2 * oy * W + 2 * ox), (int32_t)W, best, bi);
        y[t] = best;
        arg[t] = bi;
    }
}

extern "C" void nck_pool_fwd(nck_dev *d, const nck_conv *g, const float *x, float *y, int32_t *arg, int is_max) {
    int64_t total = g->N * g->C * g->OH * g->OW;
    if (total <= 0) return;
    Scope sc(d, is_max ? "max_pool" : "avg_pool", 0.0,
             4.0 * (g->N * g->C * g->H * g->W + (is_max ? 2 : 1) * total));
    const int64_t planes = g->N * g->C;
    if (is_max && g->KH == 2 && g->KW == 2 && g->sh == 2 && g->sw == 2 && g->ph == 0 && g->pw == 0 && g->W % 4 == 0 &&
        ((uintptr_t)x & 15) == 0 && small_index(planes * g->H * g->W)) {
        const int64_t items = planes * g->OH * ((g->OW + 1) / 2);
        k_maxpool2x2<<<grid_for(d, items), 256, 0, NCK_STREAM(d)>>>(x, y, arg, (uint32_t)planes, (uint32_t)g->H,
                                                                  (uint32_t)g->W, (uint32_t)g->OH, (uint32_t)g->OW);
    } else if (is_max && g->KH == 2 && g->KW == 2 && g->sh == 2 && g->sw == 2 && g->ph == 0 && g->pw == 0 &&
               g->W % 2 == 0 && ((uintptr_t)x & 7) == 0 && small_index(planes * g->H * g->W)) {
        k_maxpool2x2_w2<<<grid_for(d, total), 256, 0, NCK_STREAM(d)>>>(
            x, y, arg, (uint32_t)planes, (uint32_t)g->H, (uint32_t)g->W, (uint32_t)g->OH, (uint32_t)g->OW,
            make_fastdiv((uint32_t)g->OW), make_fastdiv((uint32_t)g->OH));
    } else if (small_index(g->N * g->C * g->H * g->W) && small_index(total))
        k_pool_fwd<uint32_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(
            *g, x, y, arg, is_max, make_fastdiv((uint32_t)g->OW), make_fastdiv((uint32_t)g->OH));
    else
        k_pool_fwd<int64_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, x, y, arg, is_max, FastDiv{1, 0, 0},
                                                                                FastDiv{1, 0, 0});
    NCK_LAUNCHED(d, 1);
}

// windows that do not overlap: each output adds its gradient to the one input it came from
template <typename I>
__global__ void k_maxpool_bwd_scatter(nck_conv g, const float *__restrict__ gy, const int32_t *__restrict__ arg,
                                      float *__restrict__ gx) {
    const I per = (I)(g.OH * g.OW), total = (I)(g.N * g.C) * per, hw = (I)(g.H * g.W);
    for (I t = blockIdx.x * (I)blockDim.x + threadIdx.x; t < total; t += (I)gridDim.x * blockDim.x)
        gx[(int64_t)(t / per) * hw + __ldg(arg + t)] += __ldg(gy + t);
}

// general windows: each input gathers from the outputs whose window holds it, in output order
template <typename I>
__global__ void k_pool_bwd_gather(nck_conv g, const float *__restrict__ gy, const int32_t *__restrict__ arg,
                                  float *__restrict__ gx, int is_max) {
    const I W = (I)g.W, H = (I)g.H;
    const I total = (I)(g.N * g.C) * H * W;
    const float inv = 1.0f / (float)(g.KH * g.KW);
    for (I t = blockIdx.x * (I)blockDim.x + threadIdx.x; t < total; t += (I)gridDim.x * blockDim.x) {
        I r = t / W, ix = t - r * W;
        I plane = r / H, iy = r - plane * H;
        int32_t self = (int32_t)(iy * W + ix);
        const float *gp = gy + (int64_t)plane * g.OH * g.OW;
        const int32_t *ap = is_max ? arg + (int64_t)plane * g.OH * g.OW : nullptr;
        float acc = gx[t];
        int64_t oy0 = (int64_t)iy + g.ph - (g.KH - 1);
        oy0 = oy0 <= 0 ? 0 : (oy0 + g.sh - 1) / g.sh;
        int64_t oy1 = ((int64_t)iy + g.ph) / g.sh;
        int64_t ox0 = (int64_t)ix + g.pw - (g.KW - 1);
        ox0 = ox0 <= 0 ? 0 : (ox0 + g.sw - 1) / g.sw;
        int64_t ox1 = ((int64_t)ix + g.pw) / g.sw;
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

// Non-overlapping windows (stride >= kernel) into a fresh gradient buffer: each input element lies in
// at most one window, so it is stored once: the window's gradient where it was the maximum (max) or
// gy / (KH*KW) (average), 0 elsewhere; the same values zero-fill plus scatter would leave.
__global__ void k_pool_bwd_set(nck_conv g, const float *__restrict__ gy, const int32_t *__restrict__ arg,
                               float *__restrict__ gx, int is_max, FastDiv divW, FastDiv divH) {
    const uint32_t W = (uint32_t)g.W, H = (uint32_t)g.H, OH = (uint32_t)g.OH, OW = (uint32_t)g.OW;
    const uint32_t total = (uint32_t)(g.N * g.C) * H * W;
    const float inv = 1.0f / (float)(g.KH * g.KW);
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = divW.div(t), ix = t - r * W, plane = divH.div(r), iy = r - plane * H;
        const uint32_t ty = iy + (uint32_t)g.ph, tx = ix + (uint32_t)g.pw;
        const uint32_t oy = ty / (uint32_t)g.sh, ox = tx / (uint32_t)g.sw;
        float v = 0.0f;
        if (ty - oy * (uint32_t)g.sh < (uint32_t)g.KH && tx - ox * (uint32_t)g.sw < (uint32_t)g.KW && oy < OH &&
            ox < OW) {
            const size_t o = (size_t)plane * OH * OW + (size_t)oy * OW + ox;
            if (is_max) v = __ldg(arg + o) == (int32_t)(iy * W + ix) ? __ldg(gy + o) : 0.0f;
            else v = __ldg(gy + o) * inv;
        }
        gx[t] = v;
    }
}

// the same for 2x2 max pooling with stride 2, no padding, width a multiple of 4: a thread stores four
// consecutive inputs of one row (two windows) with one 16-byte write
__global__ void __launch_bounds__(256) k_maxpool2x2_bwd_set(const float *__restrict__ gy,
                                                            const int32_t *__restrict__ arg, float *__restrict__ gx,
                                                            uint32_t planes, uint32_t H, uint32_t W, uint32_t OH,
                                                            uint32_t OW) {
    const uint32_t quads = W / 4, total = planes * H * quads;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = t / quads, q = t - r * quads, pl = r / H, iy = r - pl * H, oy = iy >> 1;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (oy < OH) {
            const size_t o = (size_t)pl * OH * OW + (size_t)oy * OW + 2 * q;
            const int32_t i0 = (int32_t)(iy * W + 4 * q), a0 = __ldg(arg + o), a1 = __ldg(arg + o + 1);
            const float g0 = __ldg(gy + o), g1 = __ldg(gy + o + 1);
            v.x = a0 == i0 ? g0 : 0.0f;
            v.y = a0 == i0 + 1 ? g0 : 0.0f;
            v.z = a1 == i0 + 2 ? g1 : 0.0f;
            v.w = a1 == i0 + 3 ? g1 : 0.0f;
        }
        reinterpret_cast<float4 *>(gx + (size_t)pl * H * W + (size_t)iy * W)[q] = v;
    }
}

// the same for an even width: a thread stores the two inputs of one window row with one 8-byte write
__global__ void __launch_bounds__(256) k_maxpool2x2_bwd_set_w2(const float *__restrict__ gy,
                                                               const int32_t *__restrict__ arg, float *__restrict__ gx,
                                                               uint32_t planes, uint32_t H, uint32_t W, uint32_t OH,
                                                               uint32_t OW, FastDiv dhalf, FastDiv dh) {
    const uint32_t half = W / 2, total = planes * H * half;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = dhalf.div(t), q = t - r * half, pl = dh.div(r), iy = r - pl * H, oy = iy >> 1;
        float2 v = make_float2(0.0f, 0.0f);
        if (oy < OH) {
            const size_t o = (size_t)pl * OH * OW + (size_t)oy * OW + q;
            const int32_t i0 = (int32_t)(iy * W + 2 * q), a = __ldg(arg + o);
            const float gv = __ldg(gy + o);
            v.x = a == i0 ? gv : 0.0f;
            v.y = a == i0 + 1 ? gv : 0.0f;
        }
        *reinterpret_cast<float2 *>(gx + (size_t)pl * H * W + (size_t)iy * W + 2 * q) = v;
    }
}

extern "C" void nck_pool_bwd(nck_dev *d, const nck_conv *g, const float *gy, const int32_t *arg, float *gx,
                             int is_max, int acc) {
    Scope sc(d, is_max ? "max_pool_bwd" : "avg_pool_bwd", 0.0,
             4.0 * ((is_max ? 2 : 1) * g->N * g->C * g->OH * g->OW + 2 * g->N * g->C * g->H * g->W));
    const int64_t in_total = g->N * g->C * g->H * g->W;
    if (!acc && is_max && g->KH == 2 && g->KW == 2 && g->sh == 2 && g->sw == 2 && g->ph == 0 && g->pw == 0 &&
        g->W % 4 == 0 && ((uintptr_t)gx & 15) == 0 && small_index(in_total)) {
        const int64_t items = in_total / 4;
        k_maxpool2x2_bwd_set<<<grid_for(d, items), 256, 0, NCK_STREAM(d)>>>(
            gy, arg, gx, (uint32_t)(g->N * g->C), (uint32_t)g->H, (uint32_t)g->W, (uint32_t)g->OH, (uint32_t)g->OW);
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (!acc && is_max && g->KH == 2 && g->KW == 2 && g->sh == 2 && g->sw == 2 && g->ph == 0 && g->pw == 0 &&
        g->W % 2 == 0 && ((uintptr_t)gx & 7) == 0 && small_index(in_total)) {
        k_maxpool2x2_bwd_set_w2<<<grid_for(d, in_total / 2), 256, 0, NCK_STREAM(d)>>>(
            gy, arg, gx, (uint32_t)(g->N * g->C), (uint32_t)g->H, (uint32_t)g->W, (uint32_t)g->OH, (uint32_t)g->OW,
            make_fastdiv((uint32_t)(g->W / 2)), make_fastdiv((uint32_t)g->H));
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (!acc && g->sh >= g->KH && g->sw >= g->KW && small_index(in_total)) {
        k_pool_bwd_set<<<grid_for(d, in_total), kThreads, 0, NCK_STREAM(d)>>>(
            *g, gy, arg, gx, is_max, make_fastdiv((uint32_t)g->W), make_fastdiv((uint32_t)g->H));
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (!acc) cudaMemsetAsync(gx, 0, (size_t)in_total * sizeof(float), NCK_STREAM(d));
    if (is_max && g->sh >= g->KH && g->sw >= g->KW) {
        int64_t total = g->N * g->C * g->OH * g->OW;
        if (total <= 0) return;
        if (small_index(g->N * g->C * g->H * g->W))
            k_maxpool_bwd_scatter<uint32_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx);
        else
            k_maxpool_bwd_scatter<int64_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx);
    } else {
        int64_t total = g->N * g->C * g->H * g->W;
        if (total <= 0) return;
        if (small_index(total))
            k_pool_bwd_gather<uint32_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx, is_max);
        else
            k_pool_bwd_gather<int64_t><<<grid_for(d, total), kThreads, 0, NCK_STREAM(d)>>>(*g, gy, arg, gx, is_max);
    }
    NCK_LAUNCHED(d, 1);
}
