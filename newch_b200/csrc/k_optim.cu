// Fused optimizer update: every parameter of an optimizer in one launch. The host cuts each
// parameter into chunks of NCK_OPT_CHUNK elements and keeps the (segment, chunk) tables on the
// device; block b updates chunk b with float4 loads and stores (the flat gradient / moment slices
// and the parameter allocations are 16-byte aligned), so no element searches for its segment.
// The per-element arithmetic is newch's update loop (engine/src/optim/optim.c:178-211) in the same
// order; this file is compiled without FMA contraction so each product and sum rounds as in newch.
#include <math.h>

#include "k_common.cuh"

using namespace nck;

namespace {

struct Upd {
    nck_opt_hyper h;
    // one element: w, g in; w, m, v updated (m / v untouched where the rule has none)
    __device__ __forceinline__ void operator()(float &w, float g, float *m, float *v) const {
        if (h.kind == NCK_OPT_SGD) {
            float gj = h.gs * g + h.weight_decay * w;
            if (m) {
                gj = h.momentum * *m + gj;
                *m = gj;
            }
            w = w - h.lr * gj;
        } else if (h.kind == NCK_OPT_RMSPROP) {
            float gj = h.gs * g + h.weight_decay * w;
            float a = h.beta2;
            float vj = a * *v + (1.0f - a) * gj * gj;
            *v = vj;
            float den = h.eps_inside_sqrt ? sqrtf(vj + h.eps) : sqrtf(vj) + h.eps;
            float step = gj / den;
            if (m) {
                step = h.momentum * *m + step;
                *m = step;
            }
            w = w - h.lr * step;
        } else {
            float l2 = h.kind == NCK_OPT_ADAM ? h.weight_decay : 0.0f;
            float decay = h.kind == NCK_OPT_ADAMW ? 1.0f - h.lr * h.weight_decay : 1.0f;
            float wj = w * decay;
            float gj = h.gs * g + l2 * wj;
            float mj = h.beta1 * *m + (1.0f - h.beta1) * gj;
            float vj = h.beta2 * *v + (1.0f - h.beta2) * gj * gj;
            *m = mj;
            *v = vj;
            w = wj - h.lr * (mj / h.bc1) / (sqrtf(vj / h.bc2) + h.eps);
        }
    }
};

__global__ void __launch_bounds__(256) k_optim(nck_opt_hyper h, const nck_param_seg *__restrict__ segs,
                                               const nck_opt_chunk *__restrict__ chunks,
                                               const unsigned char *__restrict__ present) {
    const nck_opt_chunk c = chunks[blockIdx.x];
    const nck_param_seg s = segs[c.seg];
    if (present && !present[s.param]) return;
    const Upd upd{h};
    float *w = s.w + c.off;
    const float *g = s.g + c.off;
    float *m = s.m ? s.m + c.off : nullptr, *v = s.v ? s.v + c.off : nullptr;
    const int n4 = c.len >> 2;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 wv = reinterpret_cast<const float4 *>(w)[i];
        const float4 gv = __ldg(reinterpret_cast<const float4 *>(g) + i);
        float4 mv = m ? reinterpret_cast<const float4 *>(m)[i] : z;
        float4 vv = v ? reinterpret_cast<const float4 *>(v)[i] : z;
        upd(wv.x, gv.x, m ? &mv.x : nullptr, v ? &vv.x : nullptr);
        upd(wv.y, gv.y, m ? &mv.y : nullptr, v ? &vv.y : nullptr);
        upd(wv.z, gv.z, m ? &mv.z : nullptr, v ? &vv.z : nullptr);
        upd(wv.w, gv.w, m ? &mv.w : nullptr, v ? &vv.w : nullptr);
        reinterpret_cast<float4 *>(w)[i] = wv;
        if (m) reinterpret_cast<float4 *>(m)[i] = mv;
        if (v) reinterpret_cast<float4 *>(v)[i] = vv;
    }
    for (int i = (n4 << 2) + threadIdx.x; i < c.len; i += blockDim.x) {
        float wj = w[i];
        upd(wj, g[i], m ? m + i : nullptr, v ? v + i : nullptr);
        w[i] = wj;
    }
}

}  // namespace

extern "C" int nck_optim_chunks(const nck_param_seg *segs, int nseg, nck_opt_chunk *chunks) {
    int k = 0;
    for (int i = 0; i < nseg; i++) {
        for (int64_t off = 0; off < segs[i].n; off += NCK_OPT_CHUNK) {
            if (chunks) {
                int64_t len = segs[i].n - off;
                chunks[k].seg = i;
                chunks[k].len = (int32_t)(len < NCK_OPT_CHUNK ? len : NCK_OPT_CHUNK);
                chunks[k].off = off;
            }
            k++;
        }
    }
    return k;
}

extern "C" void nck_optim_step(nck_dev *d, const nck_opt_hyper *h, const nck_param_seg *dsegs,
                               const nck_opt_chunk *dchunks, int nchunk, int64_t total, const unsigned char *present) {
    if (nchunk <= 0) return;
    /* Adam/AdamW: read w, g, m, v and write w, m, v (28 bytes per parameter); SGD/RMSprop less */
    double per = h->kind == NCK_OPT_ADAM || h->kind == NCK_OPT_ADAMW ? 28.0 : 20.0;
    Scope sc(d, "optim", 0.0, per * total);
    k_optim<<<nchunk, 256, 0, NCK_STREAM(d)>>>(*h, dsegs, dchunks, present);
    NCK_LAUNCHED(d, 1);
}
