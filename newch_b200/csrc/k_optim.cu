// Fused optimizer update: every parameter of an optimizer in one launch (segments table in the
// kernel parameters, elements mapped by a prefix over segment sizes). The per-element arithmetic
// is newch's update loop (engine/src/optim/optim.c:178-211) in the same order; this file is
// compiled without FMA contraction so each product and sum rounds as in newch.
#include <math.h>

#include "k_common.cuh"

using namespace nck;

namespace {

constexpr int kMaxSeg = 48;

struct SegTable {
    int n;
    int64_t start[kMaxSeg + 1];
    float *w[kMaxSeg];
    const float *g[kMaxSeg];
    float *m[kMaxSeg];
    float *v[kMaxSeg];
};

__global__ void k_optim(nck_opt_hyper h, SegTable t) {
    int64_t total = t.start[t.n];
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        int lo = 0, hi = t.n - 1;
        while (lo < hi) {  // last segment whose start <= e
            int mid = (lo + hi + 1) >> 1;
            if (t.start[mid] <= e) lo = mid;
            else hi = mid - 1;
        }
        int64_t j = e - t.start[lo];
        float *w = t.w[lo], *m = t.m[lo], *v = t.v[lo];
        float g = t.g[lo][j], wj = w[j];
        if (h.kind == NCK_OPT_SGD) {
            float gj = h.gs * g + h.weight_decay * wj;
            if (m) {
                gj = h.momentum * m[j] + gj;
                m[j] = gj;
            }
            w[j] = wj - h.lr * gj;
        } else if (h.kind == NCK_OPT_RMSPROP) {
            float gj = h.gs * g + h.weight_decay * wj;
            float a = h.beta2;
            float vj = a * v[j] + (1.0f - a) * gj * gj;
            v[j] = vj;
            float den = h.eps_inside_sqrt ? sqrtf(vj + h.eps) : sqrtf(vj) + h.eps;
            float step = gj / den;
            if (m) {
                step = h.momentum * m[j] + step;
                m[j] = step;
            }
            w[j] = wj - h.lr * step;
        } else {
            float l2 = h.kind == NCK_OPT_ADAM ? h.weight_decay : 0.0f;
            float decay = h.kind == NCK_OPT_ADAMW ? 1.0f - h.lr * h.weight_decay : 1.0f;
            wj = wj * decay;
            float gj = h.gs * g + l2 * wj;
            float mj = h.beta1 * m[j] + (1.0f - h.beta1) * gj;
            float vj = h.beta2 * v[j] + (1.0f - h.beta2) * gj * gj;
            m[j] = mj;
            v[j] = vj;
            w[j] = wj - h.lr * (mj / h.bc1) / (sqrtf(vj / h.bc2) + h.eps);
        }
    }
}

}  // namespace

extern "C" void nck_optim_step(nck_dev *d, const nck_opt_hyper *h, const nck_param_seg *segs, int nseg) {
    int64_t total = 0;
    for (int i = 0; i < nseg; i++) total += segs[i].n;
    /* Adam/AdamW: read w, g, m, v and write w, m, v (28 bytes per parameter); SGD/RMSprop less */
    double per = h->kind == NCK_OPT_ADAM || h->kind == NCK_OPT_ADAMW ? 28.0 : 20.0;
    Scope sc(d, "optim", 0.0, per * total);
    for (int s0 = 0; s0 < nseg; s0 += kMaxSeg) {
        SegTable t;
        t.n = nseg - s0 < kMaxSeg ? nseg - s0 : kMaxSeg;
        t.start[0] = 0;
        for (int i = 0; i < t.n; i++) {
            const nck_param_seg &s = segs[s0 + i];
            t.w[i] = s.w, t.g[i] = s.g, t.m[i] = s.m, t.v[i] = s.v;
            t.start[i + 1] = t.start[i] + s.n;
        }
        if (t.start[t.n] == 0) continue;
        k_optim<<<grid_for(d, t.start[t.n]), kThreads, 0, NCK_STREAM(d)>>>(*h, t);
        NCK_LAUNCHED(d, 1);
    }
}
