// Implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05.mma kind::tf32): the unfolded
// (im2col) operand is never written to memory. Producer warps gather it straight from the activation
// tensor into the 128-byte-swizzled K-major shared-memory tiles the MMA reads, splitting each value
// into its TF32 head and rest on the way in (3xTF32 mode), so no separate split pass runs either.
//
// Three products, all on NCHW fp32 tensors with groups = 1:
//   forward  D[pos][oc]  = sum over taps (c, ki, kj) of X-tap(pos) * W[oc][c, ki, kj]       -> Y (+ bias)
//   dX       D[pos][c]   = sum over taps (oc, ki, kj) of dY-tap(pos) * W[oc][c, ki, kj]     -> dX +=
//            (unit stride: dX is the convolution of dY with the flipped kernel)
//   dW       D[tap][oc]  = sum over positions (n, oy, ox) of X-tap(pos) * dY[n][oc][oy, ox] -> dW +=
// For forward and dX the 128 TMEM lanes of a tile are output positions, so epilogue stores run along
// the contiguous spatial dimension; for dW the lanes are taps (a row of dW). The dW reduction over
// positions is split across CTAs and the slices are added in a fixed order.
//
// CTA roles (416 threads, one persistent CTA per SM): warps 0-3 epilogue (tcgen05.ld, stores), warp
// 4 the MMA issuer, warps 5-12 the producers in two groups of four warps that fill alternate stages.
// A stage holds 32 K values (one 128-byte swizzle row per tile row, 4 floats per 16-byte chunk).
// Every mbarrier wait is bounded (2 s) and reports through the status word.
#include <string.h>

#include "k_common.cuh"
#include "k_tcgen05.cuh"

using namespace nck;

namespace {

using namespace tc;

constexpr int kEpiWarps = 4, kMmaWarp = 4, kProdWarp0 = 5, kProdThreads = 256;
constexpr int kIcThreads = kProdWarp0 * 32 + kProdThreads;  // 416
constexpr int kMaxTaps = 1152;

enum { IC_FWD = 0, IC_DX = 1, IC_DW = 2 };

struct IcParams {
    int mode;
    FastDiv div_pw, div_phw;  // by PW and by PH * PW
    // conv geometry (NCHW, groups 1)
    int C, OC, KH, KW, sh, sw, ph, pw, dh, dw;
    // positions: N samples of PH x PW, position (py, px) reads the gathered tensor at (py*sy, px*sx) + tap
    int64_t N;
    int PH, PW, sy, sx;
    // gathered tensor: planes of IH x IW, samples in_ns floats apart
    const float *in;
    int64_t in_ns;
    int IH, IW;
    int K;  // taps
    // second operand: weights (forward, dX) or dY (dW, samples q_ns apart)
    const float *q;
    int64_t q_ns;
    int J;     // its rows: OC (forward, dW) or C (dX)
    int q_js;  // forward: K, dX: KH*KW (row step of the weight gather)
    // output: forward / dX: out + n*out_ns + j*out_js + p; dW: out + j*K + tap
    float *out;
    int64_t out_ns, out_js;
    int accumulate;
    const float *bias;
    // dW: slices of the position range
    float *part;
    int splits;
    int64_t kper;
    int BN, stages, three;
    int64_t tiles_r, tiles_q, units;
    int *status;
};

struct Bars {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t tfull[2], tempty[2], mma_done;
    uint32_t tmem;
};

struct Tap {
    int off, dy, dx, qoff;
};

struct Unit {
    int64_t r0, j0, s, k_lo, k_hi;
};

__device__ __forceinline__ Unit unit_of(const IcParams &p, int64_t u) {
    Unit w;
    int64_t tiles = p.tiles_r * p.tiles_q, t = u % tiles;
    w.s = u / tiles;
    w.r0 = (t % p.tiles_r) * TM;
    w.j0 = (t / p.tiles_r) * p.BN;
    if (p.mode == IC_DW) {
        int64_t npos = p.N * p.PH * p.PW;
        w.k_lo = w.s * p.kper;
        w.k_hi = w.k_lo + p.kper < npos ? w.k_lo + p.kper : npos;
    } else {
        w.k_lo = 0, w.k_hi = p.K;
    }
    return w;
}

__device__ __forceinline__ void build_taps(const IcParams &p, Tap *taps) {
    const int KK = p.KH * p.KW;
    for (int k = threadIdx.x; k < p.K; k += blockDim.x) {
        Tap t;
        int ch = k / KK, kk = k - ch * KK, ki = kk / p.KW, kj = kk - ki * p.KW;
        if (p.mode == IC_DX) {  // taps (oc, ki, kj) over dY
            t.dy = p.ph - ki * p.dh;
            t.dx = p.pw - kj * p.dw;
            t.qoff = ch * p.C * KK + kk;
        } else {  // taps (c, ki, kj) over X
            t.dy = ki * p.dh - p.ph;
            t.dx = kj * p.dw - p.pw;
            t.qoff = k;
        }
        t.off = ch * p.IH * p.IW + t.dy * p.IW + t.dx;
        taps[k] = t;
    }
}

// one 16-byte chunk (4 K values) of a K-major 128-byte-swizzled tile row
__device__ __forceinline__ void put_chunk(float *tile, float *rest, int row, int q, const float (&v)[4], bool three) {
    const int idx = row * 32 + ((q ^ (row & 7)) << 2);
    // the MMA reads the fp32 value as its TF32 head (it drops the low 13 mantissa bits)
    *reinterpret_cast<float4 *>(tile + idx) = make_float4(v[0], v[1], v[2], v[3]);
    if (three) {
        *reinterpret_cast<float4 *>(rest + idx) = make_float4(tf32_rest(v[0]), tf32_rest(v[1]), tf32_rest(v[2]), tf32_rest(v[3]));
    }
}

__global__ void __launch_bounds__(kIcThreads, 1) k_convgemm(IcParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~(uintptr_t)1023);
    Bars &s = *reinterpret_cast<Bars *>(base);
    const int S = p.stages, BN = p.BN, sbq = BN * TK;
    const bool three = p.three != 0;
    float *const ring_a = reinterpret_cast<float *>(base + 1024);
    float *const ring_b = ring_a + S * kStageA;
    float *const rest_a = ring_b + S * sbq;
    float *const rest_b = rest_a + (three ? S * kStageA : 0);
    Tap *const taps = reinterpret_cast<Tap *>(rest_b + (three ? S * sbq : 0));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tcols = tmem_cols(BN);

    if (tid == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&s.full[i], kProdThreads / 2);  // the group filling that stage
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s.tfull[i], 1);
            mbar_init(&s.tempty[i], kEpiWarps);
        }
        mbar_init(&s.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    build_taps(p, taps);
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;
    const int64_t PHW = (int64_t)p.PH * p.PW, npos = p.N * PHW;

    if (warp >= kProdWarp0) {
        // ---- producers: two groups of 128 threads take alternate K steps, so two stages fill at once;
        // each thread issues all of its loads for a stage before it splits and stores any of them ----
        const int pt = tid - kProdWarp0 * 32, grp = pt >> 7, tt = pt & 127;
        int64_t it = 0;
        int pst = 0;
        uint32_t pph = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
            Unit w = unit_of(p, u);
            const int64_t ksteps = (w.k_hi - w.k_lo + TK - 1) / TK;
            // forward / dX: this thread's tile row is position r0 + tt
            int64_t row_off = 0;
            int row_y = 0, row_x = 0;
            bool row_ok = false;
            if (p.mode != IC_DW) {
                const int64_t pos = w.r0 + tt;
                row_ok = pos < npos;
                if (row_ok) {
                    const uint32_t n = p.div_phw.div((uint32_t)pos), pp = (uint32_t)pos - n * (uint32_t)PHW;
                    const uint32_t py = p.div_pw.div(pp), px = pp - py * (uint32_t)p.PW;
                    row_y = (int)py * p.sy, row_x = (int)px * p.sx;
                    row_off = (int64_t)n * p.in_ns + (int64_t)row_y * p.IW + row_x;
                }
            }
            for (int64_t ks = 0; ks < ksteps; ks++, it++) {
                // stage and phase of step it, advanced by counting (every step, the other group's too)
                const int st = pst;
                const uint32_t ph = pph;
                if (++pst == S) pst = 0, pph ^= 1;
                if ((it & 1) != grp) continue;
                if (it >= S && !(ok = mbar_wait(&s.empty[st], ph ^ 1, p.status))) break;
                const int k0 = (int)(w.k_lo + ks * TK);
                float *ta = ring_a + st * kStageA, *ra = rest_a + st * kStageA;
                float *tb = ring_b + st * sbq, *rb = rest_b + st * sbq;
                if (p.mode != IC_DW) {
                    // lane operand: row tt = a position, its 32 taps k0 .. k0 + 31
                    float v[32];
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        const int k = k0 + e;
                        float x = 0.0f;
                        if (row_ok && k < p.K) {
                            const Tap t = taps[k];
                            const int yy = row_y + t.dy, xx = row_x + t.dx;
                            if (yy >= 0 && yy < p.IH && xx >= 0 && xx < p.IW) x = __ldg(p.in + row_off + t.off);
                        }
                        v[e] = x;
                    }
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const float c4[4] = {v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]};
                        put_chunk(ta, ra, tt, q, c4, three);
                    }
                    // weights: BN rows x 8 chunks over the 128 threads
                    constexpr int kQ = kMaxBN * 8 / 128;
                    float qv[kQ][4];
#pragma unroll
                    for (int m = 0; m < kQ; m++) {
                        const int idx = tt + 128 * m, j = idx >> 3, q = idx & 7;
                        const int64_t jj = w.j0 + j;
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int k = k0 + 4 * q + e;
                            qv[m][e] = (j < BN && jj < p.J && k < p.K) ? __ldg(p.q + jj * p.q_js + taps[k].qoff) : 0.0f;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < kQ; m++) {
                        const int idx = tt + 128 * m, j = idx >> 3, q = idx & 7;
                        if (j < BN) put_chunk(tb, rb, j, q, qv[m], three);
                    }
                } else {
                    // positions k0 + 4q + e of this thread's chunk q, shared by its P and dY rows
                    const int q = tt & 7, rbase = tt >> 3;
                    int64_t in_off[4], q_off[4];
                    int py_s[4], px_s[4];
                    bool pv[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int64_t kp = (int64_t)k0 + 4 * q + e;
                        pv[e] = kp < w.k_hi;
                        const uint32_t n = pv[e] ? p.div_phw.div((uint32_t)kp) : 0u;
                        const uint32_t pp = pv[e] ? (uint32_t)kp - n * (uint32_t)PHW : 0u;
                        const uint32_t py = p.div_pw.div(pp), px = pp - py * (uint32_t)p.PW;
                        py_s[e] = (int)py * p.sy, px_s[e] = (int)px * p.sx;
                        in_off[e] = (int64_t)n * p.in_ns + (int64_t)py_s[e] * p.IW + px_s[e];
                        q_off[e] = (int64_t)n * p.q_ns + pp;
                    }
                    // lane operand: rows = taps rbase + 16 m
                    float v[8][4];
#pragma unroll
                    for (int m = 0; m < 8; m++) {
                        const int k = (int)w.r0 + rbase + 16 * m;
                        const bool kv = k < p.K;
                        const Tap t = taps[kv ? k : 0];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int yy = py_s[e] + t.dy, xx = px_s[e] + t.dx;
                            v[m][e] = (kv && pv[e] && yy >= 0 && yy < p.IH && xx >= 0 && xx < p.IW)
                                          ? __ldg(p.in + in_off[e] + t.off)
                                          : 0.0f;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < 8; m++) put_chunk(ta, ra, rbase + 16 * m, q, v[m], three);
                    // dY rows = output channels rbase + 16 m
                    constexpr int kQ = kMaxBN / 16;
                    float qv[kQ][4];
#pragma unroll
                    for (int m = 0; m < kQ; m++) {
                        const int row = rbase + 16 * m;
                        const int64_t jj = w.j0 + row;
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            qv[m][e] = (row < BN && jj < p.J && pv[e]) ? __ldg(p.q + q_off[e] + jj * PHW) : 0.0f;
                    }
#pragma unroll
                    for (int m = 0; m < kQ; m++)
                        if (rbase + 16 * m < BN) put_chunk(tb, rb, rbase + 16 * m, q, qv[m], three);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
                mbar_arrive(&s.full[st]);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ---- MMA issuer ----------------------------------------------------------------------------
            const uint32_t idesc = idesc_tf32(0, 0, BN);
            const uint64_t dA = stage_desc(smem_u32(ring_a), 0, 0), dB = stage_desc(smem_u32(ring_b), 0, 0);
            const uint32_t stA = (uint32_t)(kStageA * 4) >> 4, stB = (uint32_t)(sbq * 4) >> 4;
            const uint64_t restA = (uint64_t)((smem_u32(rest_a) - smem_u32(ring_a)) >> 4);
            const uint64_t restB = (uint64_t)((smem_u32(rest_b) - smem_u32(ring_b)) >> 4);
            int st = 0;
            uint32_t ph = 0;
            int64_t it = 0, local = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, local++) {
                Unit w = unit_of(p, u);
                const int64_t ksteps = (w.k_hi - w.k_lo + TK - 1) / TK;
                const int acc = (int)(local & 1);
                if (local >= 2 && !(ok = mbar_wait(&s.tempty[acc], (uint32_t)(((local >> 1) & 1) ^ 1), p.status)))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + (uint32_t)acc * (tcols / 2);
                for (int64_t ks = 0; ks < ksteps; ks++, it++) {
                    if (!(ok = mbar_wait(&s.full[st], ph, p.status))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    // descriptors by addition: only the start-address field moves
                    const uint64_t a0 = dA + (uint64_t)(st * stA), b0 = dB + (uint64_t)(st * stB);
#pragma unroll
                    for (int k = 0; k < TK / 8; k++) {
                        const uint32_t accum = (ks > 0 || k > 0) ? 1u : 0u;
                        const uint64_t ak = a0 + (uint64_t)(2 * k), bk = b0 + (uint64_t)(2 * k);
                        mma_tf32(d, ak, bk, idesc, accum);
                        if (three) {
                            mma_tf32(d, ak, bk + restB, idesc, 1u);
                            mma_tf32(d, ak + restA, bk, idesc, 1u);
                        }
                    }
                    mma_commit(&s.empty[st]);
                    if (++st == S) st = 0, ph ^= 1;
                }
                if (ok) mma_commit(&s.tfull[acc]);
            }
            mma_commit(&s.mma_done);
            mbar_wait(&s.mma_done, 0, p.status);
        }
    } else {
        // ---- epilogue ---------------------------------------------------------------------------------
        int64_t local = 0;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x, local++) {
            Unit w = unit_of(p, u);
            const int acc = (int)(local & 1);
            if (!mbar_wait(&s.tfull[acc], (uint32_t)((local >> 1) & 1), p.status)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int64_t i = w.r0 + warp * 32 + lane;
            bool live;
            float *lane_base;
            int64_t js;
            bool add = p.accumulate != 0;
            if (p.mode != IC_DW) {
                live = i < npos;
                int64_t n = live ? i / PHW : 0;
                lane_base = p.out + n * p.out_ns + (i - n * PHW);
                js = p.out_js;
            } else {
                live = i < p.K;
                float *o = p.splits > 1 ? p.part + w.s * (int64_t)p.J * p.K : p.out;
                add = p.splits > 1 ? false : add;
                lane_base = o + i;
                js = p.K;
            }
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t rr[16];
                tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)acc * (tcols / 2) + (uint32_t)c0, rr);
                if (!live) continue;
#pragma unroll
                for (int jj = 0; jj < 16; jj++) {
                    const int64_t j = w.j0 + c0 + jj;
                    if (j < p.J) {
                        float v = __uint_as_float(rr[jj]);
                        if (p.bias) v = v + __ldg(p.bias + j);
                        float *dst = lane_base + j * js;
                        *dst = add ? *dst + v : v;
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.tempty[acc]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
}

// dW += sum of the position slices' partial rows, slices in order
__global__ void k_convgemm_combine(const float *__restrict__ part, int splits, int64_t n, float *__restrict__ gw) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int k = 0; k < splits; k++) s += part[k * n + i];
        gw[i] += s;
    }
}

int pick_bn_ic(int64_t j) {
    int best = 128;
    int64_t best_cost = INT64_MAX;
    for (int bn = 32; bn <= kMaxBN; bn += 32) {
        int64_t tiles = (j + bn - 1) / bn, cost = tiles * (bn + 32);
        if (cost < best_cost) best_cost = cost, best = bn;
    }
    return best;
}

size_t tail_bytes(int K) { return (size_t)K * sizeof(Tap); }

int stages_for(int bn, bool three, int K) {
    size_t per = (size_t)(kStageA + bn * TK) * 4 * (three ? 2 : 1);
    size_t room = kSmemLimit - 2048 - tail_bytes(K);
    size_t n = room / per;
    return (int)(n > (size_t)kMaxStages ? kMaxStages : n);
}

}  // namespace

// Implicit-GEMM convolution (mode 0 forward, 1 dX, 2 dW). Returns 0 without launching anything when
// the convolution is not one it handles (groups != 1, dX with a stride, too many taps, the FFMA GEMM
// mode), and the caller takes the unfolded path.
extern "C" int nck_conv_implicit_supported(const nck_dev *d, int mode, const nck_conv *g) {
    if (!d->conv_implicit || d->gemm_mode == NCK_GEMM_FFMA || g->G != 1) return 0;
    if (mode == IC_DX && (g->sh != 1 || g->sw != 1)) return 0;
    const int64_t KK = g->KH * g->KW, L = g->OH * g->OW, HW = g->H * g->W;
    const int64_t K = (mode == IC_DX ? g->OC : g->C) * KK;
    if (K <= 0 || K > kMaxTaps || g->N <= 0 || L <= 0) return 0;
    if (g->C * HW > INT32_MAX / 2 || g->OC * L > INT32_MAX / 2 || g->C * KK * g->OC > INT32_MAX / 2) return 0;
    const int64_t npos = mode == IC_DX ? g->N * HW : g->N * L;
    if (npos >= ((int64_t)1 << 31)) return 0; /* positions index in 32 bits */
    return stages_for(pick_bn_ic(mode == IC_DX ? g->C : g->OC), d->gemm_mode == NCK_GEMM_3XTF32, (int)K) >= 2;
}

extern "C" int nck_conv_implicit(nck_dev *d, int mode, const nck_conv *g, const float *in, const float *q, float *out,
                                 const float *bias) {
    if (!nck_conv_implicit_supported(d, mode, g)) return 0;
    const int64_t KK = g->KH * g->KW, L = g->OH * g->OW, HW = g->H * g->W;
    const int64_t K = (mode == IC_DX ? g->OC : g->C) * KK;
    const bool three = d->gemm_mode == NCK_GEMM_3XTF32;

    IcParams p;
    memset(&p, 0, sizeof p);
    p.mode = mode;
    p.C = (int)g->C, p.OC = (int)g->OC, p.KH = (int)g->KH, p.KW = (int)g->KW;
    p.sh = g->sh, p.sw = g->sw, p.ph = g->ph, p.pw = g->pw, p.dh = g->dh, p.dw = g->dw;
    p.N = g->N, p.K = (int)K, p.three = three, p.status = d->status, p.in = in, p.q = q, p.out = out;
    const int64_t sms = d->sm_count > 0 ? d->sm_count : 148;
    if (mode == IC_FWD || mode == IC_DW) {
        p.PH = (int)g->OH, p.PW = (int)g->OW, p.sy = g->sh, p.sx = g->sw;
        p.IH = (int)g->H, p.IW = (int)g->W, p.in_ns = g->C * HW;
        p.J = (int)g->OC;
    } else {
        p.PH = (int)g->H, p.PW = (int)g->W, p.sy = 1, p.sx = 1;
        p.IH = (int)g->OH, p.IW = (int)g->OW, p.in_ns = g->OC * L;
        p.J = (int)g->C;
    }
    if (g->N * (int64_t)p.PH * p.PW >= ((int64_t)1 << 31)) return 0;  /* positions index in 32 bits */
    p.div_pw = make_fastdiv((uint32_t)p.PW);
    p.div_phw = make_fastdiv((uint32_t)(p.PH * p.PW));
    p.BN = pick_bn_ic(p.J);
    p.stages = stages_for(p.BN, three, p.K);
    if (p.stages < 2) return 0;
    p.tiles_q = (p.J + p.BN - 1) / p.BN;
    const int64_t npos = g->N * p.PH * p.PW;
    if (mode == IC_FWD) {
        p.q_js = p.K, p.out_ns = g->OC * L, p.out_js = L, p.bias = bias, p.accumulate = 0;
        p.tiles_r = (npos + TM - 1) / TM, p.splits = 1;
    } else if (mode == IC_DX) {
        p.q_js = (int)KK, p.out_ns = g->C * HW, p.out_js = HW, p.accumulate = 1;
        p.tiles_r = (npos + TM - 1) / TM, p.splits = 1;
    } else {
        p.q_ns = g->OC * L, p.accumulate = 1;
        p.tiles_r = (p.K + TM - 1) / TM;
        const int64_t tiles = p.tiles_r * p.tiles_q, wsz = (int64_t)p.J * p.K;
        int64_t splits = (sms + tiles - 1) / tiles;
        const int64_t maxs = (int64_t)(d->scratch_bytes / sizeof(float)) / wsz;
        if (splits > maxs) splits = maxs;
        if (splits > (npos + TK - 1) / TK) splits = (npos + TK - 1) / TK;
        if (splits < 1) splits = 1;
        p.kper = ((npos + splits - 1) / splits + TK - 1) / TK * TK;
        p.splits = (int)((npos + p.kper - 1) / p.kper);
        p.part = (float *)d->scratch;
    }
    p.units = p.tiles_r * p.tiles_q * (mode == IC_DW ? p.splits : 1);

    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(k_convgemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        attr_done = 1;
    }
    const size_t smem = 2048 + (size_t)p.stages * (kStageA + p.BN * TK) * 4 * (three ? 2 : 1) + tail_bytes(p.K);
    static const char *names[3] = {"conv_igemm_fwd", "conv_igemm_dx", "conv_igemm_dw"};
    const double flops = 2.0 * g->N * L * g->OC * g->C * KK;
    const double bytes = mode == IC_FWD ? 4.0 * (g->N * g->C * HW + g->N * g->OC * L + g->OC * g->C * KK)
                       : mode == IC_DX ? 4.0 * (g->N * g->OC * L + 2.0 * g->N * g->C * HW + g->OC * g->C * KK)
                                       : 4.0 * (g->N * g->C * HW + g->N * g->OC * L + 2.0 * g->OC * g->C * KK);
    Scope sc(d, names[mode], flops, bytes);
    const unsigned grid = (unsigned)(p.units < sms ? p.units : sms);
    k_convgemm<<<grid, kIcThreads, smem, NCK_STREAM(d)>>>(p);
    if (cudaGetLastError() != cudaSuccess) {
        *(volatile int *)d->status_host = NCK_ERR_LAUNCH;
        return 1;
    }
    int launched = 1;
    if (mode == IC_DW && p.splits > 1) {
        const int64_t wsz = (int64_t)p.J * p.K;
        k_convgemm_combine<<<grid_for(d, wsz), kThreads, 0, NCK_STREAM(d)>>>(p.part, p.splits, wsz, out);
        launched++;
    }
    NCK_LAUNCHED(d, launched);
    return 1;
}
