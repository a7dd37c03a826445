// Stride-1 convolutions (groups 1) as tap-shifted GEMMs on the 5th-generation tensor cores.
//
// Layout. An activation x [N][C][H][W] is packed once into a position-major matrix over the padded
// grid: row v = n*Hp*Wp + h'*Wp + w' (Hp = H + 2ph, Wp = W + 2pw) holds the channels of padded pixel
// (h', w'), zero on the border and in the channel padding up to Cp (a multiple of 32). The output
// pixel (oh, ow) is computed on the same grid, at row v = n*Hp*Wp + oh*Wp + ow, and filter tap
// (ki, kj) reads row v + ki*dh*Wp + kj*dw. Each tap is therefore one shift of the row coordinate of an
// ordinary TMA tile load: no unfolded copy is ever written. Rows whose (oh, ow) falls outside the
// output are computed and dropped; in the output gradient packed on the same grid they are zero.
//
//   forward  D[v][oc] = sum_tap sum_c  X~[v + s(tap)][c]  * Wf[oc][tap][c]      (both K-major)
//   dX       D[u][c]  = sum_tap sum_oc G~[u - s(tap)][oc] * Wx[c][tap][oc]      (both K-major)
//   dW       D[tap*Cp + c][oc] = sum_v X~[v + s(tap)][c] * G~[v][oc]           (both MN-major)
//
// The loads that run off either end of the packed matrix (negative rows in dX, rows past the end) are
// filled with zeros by the TMA unit; only pixels whose taps stay inside their own image are kept.
//
// Kernel: persistent CTAs, one per SM, warp-specialised like the plain GEMM: warps 0-3 epilogue
// (tcgen05.ld, then NCHW stores of the valid pixels), warp 4 the TMA loader, warp 5 the MMA issuer,
// two accumulators in TMEM. In 3xTF32 mode the packing kernels already wrote the TF32 remainders of
// every operand (a second plane of the same shape); the loader stages both planes, the Q remainder
// right after the Q head so that the two form one operand twice as wide, and the MMA thread issues
// two MMAs per K step: A_head x [Q_head | Q_rest] into a 2*BN-wide accumulator, then A_rest x Q_head
// into its first half. The epilogue adds the two halves. (The tensor core reads an fp32 operand as
// its TF32 head by dropping the low 13 mantissa bits.) Every mbarrier wait is bounded (2 s), records an error in
// the status word when it gives up, and the CTA drains its copies and MMAs and frees TMEM before
// returning.
#include <string.h>

#include "k_common.cuh"
#include "k_tcgen05.cuh"

using namespace nck;

namespace {

using namespace tc;

constexpr int kEpiWarps = 4, kLoadWarp = 4, kMmaWarp = 5, kThreadsCt = 6 * 32;
enum { MODE_FWD = 0, MODE_DX = 1, MODE_DW = 2 };

struct CtParams {
    int64_t R, Cq;        // accumulator rows (pixels of the padded grid, or tap x channel for dW), columns
    int64_t K;            // dW: positions summed (rows of the packed matrices)
    int BN, stages;
    int64_t tiles_r, tiles_q, units;
    int ksteps;           // forward / dX: K steps per tile (taps x 32-channel blocks)
    int CB;               // 32-channel blocks per tap of the P operand
    int KW, T;            // kernel width, taps
    int offh, offw;       // row shift of one kernel row (dh * Wp) and of one kernel column (dw)
    int sgn;              // +1: tap rows at v + shift (forward, dW); -1: at v - shift (dX)
    int64_t kper;         // dW: positions per reduction slice
    int splits;
    FastDiv dimg, drow;   // Hp * Wp, Wp
    int eh, ew, DH, DW;   // destination pixel (h' - eh, w' - ew), kept inside [0, DH) x [0, DW)
    int64_t out_img, out_ch;
    float *out;
    const float *bias;
    int acc;
    float *part;          // dW partial tiles [slice][Cq][R]
    int *status;
};

struct Bars {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t tfull[2], tempty[2], mma_done;
    uint32_t tmem;
};

struct CtUnit {
    int64_t r0, q0, sl, v0;
    int steps;
};

template <int MODE>
__device__ __forceinline__ CtUnit ct_unit(const CtParams &p, int64_t u) {
    CtUnit w;
    const int64_t tiles = p.tiles_r * p.tiles_q, t = u % tiles;
    w.sl = u / tiles;
    // column tiles of one row tile are neighbours, so they read the same P rows at about the same time
    w.r0 = (t / p.tiles_q) * TM;
    w.q0 = (t % p.tiles_q) * p.BN;
    if (MODE == MODE_DW) {
        w.v0 = w.sl * p.kper;
        int64_t v1 = w.v0 + p.kper < p.K ? w.v0 + p.kper : p.K;
        w.steps = (int)((v1 - w.v0 + TK - 1) / TK);
    } else {
        w.v0 = 0;
        w.steps = p.ksteps;
    }
    return w;
}

template <int MODE, bool THREE>
__global__ void __launch_bounds__(kThreadsCt, 1)
    k_convtap(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmPr,
              const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQr, CtParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~(uintptr_t)1023);
    Bars &s = *reinterpret_cast<Bars *>(base);
    // per stage: P head, P rest (3xTF32), and Q head followed by Q rest (3xTF32)
    const int S = p.stages, BN = p.BN, sbq = BN * TK, sbq2 = THREE ? 2 * sbq : sbq;
    float *const ring_a = reinterpret_cast<float *>(base + 1024);
    float *const rest_a = ring_a + S * kStageA;  // 3xTF32 only
    float *const ring_b = rest_a + (THREE ? S * kStageA : 0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // accumulator columns per tile: [A_h Q_h + A_r Q_h | A_h Q_r] in 3xTF32 mode. (A separate
    // accumulator for A_r Q_h was measured slower on B200: more tensor-memory traffic per MMA.)
    const int AW = THREE ? 2 * BN : BN;
    const uint32_t tcols = tmem_cols(AW);
    const uint32_t stage_bytes = (uint32_t)(TM + BN) * TK * 4 * (THREE ? 2 : 1);
    constexpr bool MN = MODE == MODE_DW;

    if (tid == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s.tfull[i], 1);
            mbar_init(&s.tempty[i], kEpiWarps);
        }
        mbar_init(&s.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;

    if (warp == kLoadWarp) {
        if (lane == 0) {
            // ---- loader ------------------------------------------------------------------------------
            int64_t it = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                const CtUnit w = ct_unit<MODE>(p, u);
                if (MODE != MODE_DW) {
                    // K step = (tap, 32-channel block); the Q column of step t is 32 t
                    int cb = 0, ki = 0, kj = 0;
                    for (int t = 0; t < w.steps; t++, it++) {
                        if (it >= S && !(ok = mbar_wait(&s.empty[st], ph ^ 1, p.status))) break;
                        mbar_expect_tx(&s.full[st], stage_bytes);
                        const int row = (int)w.r0 + p.sgn * (ki * p.offh + kj * p.offw);
                        tma_2d(ring_a + st * kStageA, &tmP, cb * TK, row, &s.full[st]);
                        tma_2d(ring_b + st * sbq2, &tmQ, t * TK, (int)w.q0, &s.full[st]);
                        if (THREE) {
                            tma_2d(rest_a + st * kStageA, &tmPr, cb * TK, row, &s.full[st]);
                            tma_2d(ring_b + st * sbq2 + sbq, &tmQr, t * TK, (int)w.q0, &s.full[st]);
                        }
                        if (++st == S) st = 0, ph ^= 1;
                        if (++cb == p.CB) {
                            cb = 0;
                            if (++kj == p.KW) kj = 0, ki++;
                        }
                    }
                } else {
                    // the tile's 128 rows are four 32-row blocks, each one (tap, channel block): its own
                    // channel column and row shift; blocks past the last tap load any valid tile (their
                    // rows are never stored)
                    int px[TM / 32], poff[TM / 32];
#pragma unroll
                    for (int j = 0; j < TM / 32; j++) {
                        int bi = (int)(w.r0 / 32) + j, tap = bi / p.CB, cb = bi - tap * p.CB;
                        if (tap >= p.T) tap = 0, cb = 0;
                        px[j] = cb * 32;
                        poff[j] = (tap / p.KW) * p.offh + (tap % p.KW) * p.offw;
                    }
                    int v = (int)w.v0;
                    for (int t = 0; t < w.steps; t++, it++, v += TK) {
                        if (it >= S && !(ok = mbar_wait(&s.empty[st], ph ^ 1, p.status))) break;
                        mbar_expect_tx(&s.full[st], stage_bytes);
#pragma unroll
                        for (int j = 0; j < TM / 32; j++) {
                            tma_2d(ring_a + st * kStageA + j * 1024, &tmP, px[j], v + poff[j], &s.full[st]);
                            if (THREE) tma_2d(rest_a + st * kStageA + j * 1024, &tmPr, px[j], v + poff[j], &s.full[st]);
                        }
                        for (int j = 0; j < BN / 32; j++) {
                            tma_2d(ring_b + st * sbq2 + j * 1024, &tmQ, (int)w.q0 + 32 * j, v, &s.full[st]);
                            if (THREE) tma_2d(ring_b + st * sbq2 + sbq + j * 1024, &tmQr, (int)w.q0 + 32 * j, v, &s.full[st]);
                        }
                        if (++st == S) st = 0, ph ^= 1;
                    }
                }
            }
            // no copy may still be landing in shared memory when the CTA exits
            int64_t first = it > S ? it - S : 0;
            for (int64_t j = first; j < it; j++)
                if (!mbar_wait(&s.full[j % S], (uint32_t)((j / S) & 1), p.status)) break;
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ---- MMA issuer ----------------------------------------------------------------------------
            // the Q head and rest are adjacent: one operand 2*BN wide (K-major: 2*BN rows of 128 B;
            // MN-major: 2*BN/32 blocks of 4 KiB, the block stride of the descriptor)
            const uint32_t idesc = idesc_tf32(MN, MN, BN), idesc2 = idesc_tf32(MN, MN, 2 * BN);
            const uint64_t dA = stage_desc(smem_u32(ring_a), MN, 0), dB = stage_desc(smem_u32(ring_b), MN, 0);
            const uint32_t stA = (uint32_t)(kStageA * 4) >> 4, stB = (uint32_t)(sbq2 * 4) >> 4;
            const uint32_t kstep = MN ? 64u : 2u;  // 8 K rows (MN-major) or 32 B along the row (K-major)
            const uint64_t restA = (uint64_t)((smem_u32(rest_a) - smem_u32(ring_a)) >> 4);
            int64_t local = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, local++) {
                const CtUnit w = ct_unit<MODE>(p, u);
                const int acc = (int)(local & 1);
                if (local >= 2 && !(ok = mbar_wait(&s.tempty[acc], (uint32_t)(((local >> 1) & 1) ^ 1), p.status)))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + (uint32_t)acc * (tcols / 2);
                for (int t = 0; t < w.steps; t++) {
                    if (!(ok = mbar_wait(&s.full[st], ph, p.status))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint64_t a0 = dA + (uint64_t)(st * stA), b0 = dB + (uint64_t)(st * stB);
#pragma unroll
                    for (int k = 0; k < TK / 8; k++) {
                        const uint32_t accum = (t > 0 || k > 0) ? 1u : 0u;
                        const uint64_t ak = a0 + (uint64_t)(k * kstep), bk = b0 + (uint64_t)(k * kstep);
                        if (THREE) {
                            mma_tf32(d, ak, bk, idesc2, accum);     // [A_h Q_h | A_h Q_r]
                            mma_tf32(d, ak + restA, bk, idesc, 1u);  // += A_r Q_h in the first half
                        } else {
                            mma_tf32(d, ak, bk, idesc, accum);
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
    } else if (warp < kEpiWarps) {
        // ---- epilogue: accumulator lane i = row r0 + 32 * warp + lane ----------------------------------
        int64_t local = 0;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x, local++) {
            const CtUnit w = ct_unit<MODE>(p, u);
            const int acc = (int)(local & 1);
            if (!mbar_wait(&s.tfull[acc], (uint32_t)((local >> 1) & 1), p.status)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int64_t i = w.r0 + warp * 32 + lane;
            float *dst;
            int64_t jstride;
            bool live = i < p.R;
            if (MODE == MODE_DW) {
                dst = p.part + w.sl * p.R * p.Cq + i;
                jstride = p.R;
            } else {
                // pixel of the padded grid -> destination pixel, kept when inside [0, DH) x [0, DW)
                const uint32_t v = live ? (uint32_t)i : 0u;
                const uint32_t n = p.dimg.div(v), rem = v - n * p.dimg.d;
                const uint32_t hh = p.drow.div(rem), ww = rem - hh * p.drow.d;
                const int dh = (int)hh - p.eh, dw = (int)ww - p.ew;
                live = live && dh >= 0 && dh < p.DH && dw >= 0 && dw < p.DW;
                dst = p.out + (int64_t)n * p.out_img + (int64_t)dh * p.DW + dw;
                jstride = p.out_ch;
            }
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16], r2[16];
                const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)acc * (tcols / 2) + (uint32_t)c0;
                tmem_ld16_nw(taddr, r);
                if (THREE) tmem_ld16_nw(taddr + (uint32_t)BN, r2);
                tmem_wait_ld(r);
                if (THREE) tmem_regs_after_wait(r2);
                const int64_t jb = w.q0 + c0;
                const int nj = p.Cq - jb < 16 ? (int)(p.Cq - jb) : 16;
                if (!live || nj <= 0) continue;
                float v[16];
#pragma unroll
                for (int jj = 0; jj < 16; jj++)
                    v[jj] = THREE ? __uint_as_float(r[jj]) + __uint_as_float(r2[jj]) : __uint_as_float(r[jj]);
                float *o = dst + jb * jstride;
                // every load of the chunk is issued before the first store, so their latencies overlap
                if (MODE == MODE_FWD && p.bias) {
                    float bv[16];
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) bv[jj] = jj < nj ? p.bias[jb + jj] : 0.0f;
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += bv[jj];
                } else if (MODE == MODE_DX && p.acc) {
                    float old[16];
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) old[jj] = jj < nj ? o[jj * jstride] : 0.0f;
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += old[jj];
                }
#pragma unroll
                for (int jj = 0; jj < 16; jj++)
                    if (jj < nj) o[jj * jstride] = v[jj];
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

// gw[oc][c][tap] (+)= sum over slices of part[slice][oc][tap * Cp + c]. Consecutive threads take
// consecutive channels, so the reads of every slice are coalesced; four running sums keep four loads
// in flight, and they are added in a fixed order.
__global__ void k_tap_dw_combine(const float *__restrict__ part, float *__restrict__ gw, int splits, int64_t R,
                                 int64_t Cq, int C, int T, int Cp, int acc) {
    const int64_t total = Cq * C * T, slice = R * Cq;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t oc = e / ((int64_t)C * T), rem = e - oc * C * T;
        const int tap = (int)(rem / C), c = (int)(rem - (int64_t)tap * C);
        const float *src = part + oc * R + (int64_t)tap * Cp + c;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        int k = 0;
        for (; k + 4 <= splits; k += 4) {
            s0 += __ldcg(src + (int64_t)k * slice);
            s1 += __ldcg(src + (int64_t)(k + 1) * slice);
            s2 += __ldcg(src + (int64_t)(k + 2) * slice);
            s3 += __ldcg(src + (int64_t)(k + 3) * slice);
        }
        for (; k < splits; k++) s0 += __ldcg(src + (int64_t)k * slice);
        const float s = (s0 + s1) + (s2 + s3);
        const int64_t o = (oc * C + c) * T + tap;
        gw[o] = acc ? gw[o] + s : s;
    }
}

// dst[v][k] for 128 rows v and 32 columns k per block: src[n][k][h' - eh][w' - ew] where that pixel
// exists, else 0 (border, channel padding). Staged through shared memory so that both the NCHW
// reads (along w) and the row-major writes (along k, 16 bytes per thread) are coalesced; the
// remainder plane follows. With 256 threads a thread reads one row v for every other k, so the row's
// image coordinates are divided out once.
__global__ void __launch_bounds__(256) k_tap_pack(const float *__restrict__ src, float *__restrict__ dst,
                                                  float *__restrict__ rest, int64_t Nv, int C, int Kp, int Hs,
                                                  int Ws, FastDiv dimg, FastDiv drow, int eh, int ew,
                                                  float *__restrict__ csum) {
    __shared__ float tile[128][33];
    __shared__ float red[8][32];
    const int64_t v0 = blockIdx.x * 128ll;
    const int k0 = blockIdx.y * 32;
    const int64_t plane = (int64_t)Hs * Ws, img = (int64_t)C * plane;
    {
        const int r = threadIdx.x & 127, kb = threadIdx.x >> 7;  // rows r, columns kb, kb + 2, ...
        const int64_t v = v0 + r;
        const float *s = nullptr;
        if (v < Nv) {
            const uint32_t n = dimg.div((uint32_t)v), rem = (uint32_t)v - n * dimg.d;
            const uint32_t hh = drow.div(rem), ww = rem - hh * drow.d;
            const int h = (int)hh - eh, w = (int)ww - ew;
            if (h >= 0 && h < Hs && w >= 0 && w < Ws) s = src + n * img + (int64_t)h * Ws + w;
        }
#pragma unroll 4
        for (int k = kb; k < 32; k += 2) tile[r][k] = (s && k0 + k < C) ? __ldg(s + (k0 + k) * plane) : 0.0f;
    }
    __syncthreads();
    if (csum) {
        // this block's sum of each of its 32 columns (rows in a fixed order: 16 per warp, then 8 warps)
        const int k = threadIdx.x & 31, wv = threadIdx.x >> 5;
        float a = 0.0f;
#pragma unroll
        for (int r = 0; r < 16; r++) a += tile[wv * 16 + r][k];
        red[wv][k] = a;
        __syncthreads();
        if (threadIdx.x < 32) {
            float t = red[0][threadIdx.x];
            for (int j = 1; j < 8; j++) t += red[j][threadIdx.x];
            csum[(int64_t)blockIdx.x * Kp + k0 + threadIdx.x] = t;
        }
    }
    for (int e = threadIdx.x; e < 8 * 128; e += blockDim.x) {
        const int q = e & 7, r = e >> 3;  // 16-byte quarter q of row r
        const int64_t v = v0 + r;
        if (v >= Nv) break;
        const float4 x = make_float4(tile[r][4 * q], tile[r][4 * q + 1], tile[r][4 * q + 2], tile[r][4 * q + 3]);
        *reinterpret_cast<float4 *>(dst + v * Kp + k0 + 4 * q) = x;
        if (rest) *reinterpret_cast<float4 *>(rest + v * Kp + k0 + 4 * q) = tf32_rest4(x);
    }
}

// forward weights dst[oc][tap][c] (tr 0, c < Cp) or dX weights dst[c][tap][oc] (tr 1, oc < OCp) from
// w[oc][c][tap]; padding columns are zero; the remainder plane follows
__global__ void k_tap_pack_w(const float *__restrict__ w, float *__restrict__ dst, float *__restrict__ rest, int OC,
                             int C, int T, int Kp, int tr) {
    const int rows = tr ? C : OC;
    const int64_t total = (int64_t)rows * T * Kp;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / ((int64_t)T * Kp)), rem = (int)(e - (int64_t)r * T * Kp);
        const int tap = rem / Kp, k = rem - tap * Kp;
        const int oc = tr ? k : r, c = tr ? r : k;
        const float x = (oc < OC && c < C) ? w[((int64_t)oc * C + c) * T + tap] : 0.0f;
        dst[e] = x;
        if (rest) rest[e] = tf32_rest(x);
    }
}

template <int MODE, bool THREE>
bool ct_smem_attr() {
    static int done = 0;
    if (done) return true;
    if (cudaFuncSetAttribute(k_convtap<MODE, THREE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    done = 1;
    return true;
}

template <int MODE>
bool ct_launch(nck_dev *d, bool three, unsigned grid, size_t smem, const CUtensorMap *m, const CtParams &p) {
    if (three) {
        if (!ct_smem_attr<MODE, true>()) return false;
        k_convtap<MODE, true><<<grid, kThreadsCt, smem, NCK_STREAM(d)>>>(m[0], m[1], m[2], m[3], p);
    } else {
        if (!ct_smem_attr<MODE, false>()) return false;
        k_convtap<MODE, false><<<grid, kThreadsCt, smem, NCK_STREAM(d)>>>(m[0], m[1], m[2], m[3], p);
    }
    return true;
}

// Q tile width: the fewest wasted columns, counting ~32 columns of per-tile overhead
int ct_pick_bn(int64_t cq) {
    int best = 128;
    int64_t best_cost = INT64_MAX;
    for (int bn = 32; bn <= kMaxBN; bn += 32) {
        int64_t tiles = (cq + bn - 1) / bn, cost = tiles * (bn + 32);
        if (cost < best_cost) best_cost = cost, best = bn;
    }
    return best;
}

int64_t round32(int64_t x) { return (x + 31) / 32 * 32; }

}  // namespace

extern "C" int nck_convtap_plan(const nck_dev *d, const nck_conv *g, nck_tapgeom *t) {
    if (!d->conv_tap || d->gemm_mode == NCK_GEMM_FFMA || g->G != 1 || g->sh != 1 || g->sw != 1) return 0;
    nck_tapgeom r;
    r.Hp = g->H + 2 * (int64_t)g->ph, r.Wp = g->W + 2 * (int64_t)g->pw;
    r.Nv = g->N * r.Hp * r.Wp;
    r.Cp = round32(g->C), r.OCp = round32(g->OC), r.T = g->KH * g->KW;
    r.planes = d->gemm_mode == NCK_GEMM_3XTF32 ? 2 : 1;
    // every TMA row coordinate (a row plus or minus the largest tap shift) fits an int32
    const int64_t shift = (g->KH - 1) * g->dh * r.Wp + (g->KW - 1) * g->dw;
    if (r.Nv + shift + 2 * TM >= ((int64_t)1 << 31) || r.T * r.Cp >= ((int64_t)1 << 31) ||
        r.T * r.OCp >= ((int64_t)1 << 31) || r.Hp * r.Wp >= ((int64_t)1 << 31))
        return 0;
    if (t) *t = r;
    return 1;
}

extern "C" void nck_tap_pack(nck_dev *d, const float *src, int64_t N, int64_t C, int64_t Hs, int64_t Ws,
                             const nck_tapgeom *t, int eh, int ew, int64_t Kp, float *dst, float *colsum) {
    if (t->Nv <= 0) return;
    Scope sc(d, "conv_tap_pack", 0.0, 4.0 * (N * C * Hs * Ws + (double)t->planes * t->Nv * Kp));
    const int64_t blocks = (t->Nv + 127) / 128;
    dim3 grid((unsigned)blocks, (unsigned)(Kp / 32));
    float *rest = t->planes == 2 ? dst + t->Nv * Kp : nullptr;
    // per-block column sums go to scratch, consumed by the column sum right behind (stream order)
    float *csum = colsum && (size_t)(blocks * Kp) * sizeof(float) <= d->scratch_bytes ? (float *)d->scratch : nullptr;
    k_tap_pack<<<grid, 256, 0, NCK_STREAM(d)>>>(src, dst, rest, t->Nv, (int)C, (int)Kp, (int)Hs, (int)Ws,
                                                 make_fastdiv((uint32_t)(t->Hp * t->Wp)),
                                                 make_fastdiv((uint32_t)t->Wp), eh, ew, csum);
    NCK_LAUNCHED(d, 1);
    if (csum) nck_colsum_ld(d, csum, Kp, colsum, blocks, C);  // gb[c] += the blocks' sums, in order
}

extern "C" int nck_tap_pack_colsum_ok(const nck_dev *d, const nck_tapgeom *t, int64_t Kp) {
    return (size_t)(((t->Nv + 127) / 128) * Kp) * sizeof(float) <= d->scratch_bytes;
}

extern "C" void nck_tap_pack_w(nck_dev *d, const nck_conv *g, const nck_tapgeom *t, const float *w, float *dst,
                               int tr) {
    const int64_t Kp = tr ? t->OCp : t->Cp, rows = tr ? g->C : g->OC, n = rows * t->T * Kp;
    float *rest = t->planes == 2 ? dst + n : nullptr;
    k_tap_pack_w<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(w, dst, rest, (int)g->OC, (int)g->C, (int)t->T,
                                                                 (int)Kp, tr);
    NCK_LAUNCHED(d, 1);
}

extern "C" int nck_convtap(nck_dev *d, int mode, const nck_conv *g, const nck_tapgeom *t, const float *P,
                           const float *Q, float *out, const float *bias, int acc) {
    if (!nck_convtap_plan(d, g, nullptr) || g->N <= 0) return 0;
    const bool three = t->planes == 2;
    const int64_t Nv = t->Nv, Cp = t->Cp, OCp = t->OCp, T = t->T;
    CtParams p;
    memset(&p, 0, sizeof p);
    p.KW = (int)g->KW, p.T = (int)T;
    p.offh = (int)(g->dh * t->Wp), p.offw = g->dw;
    p.dimg = make_fastdiv((uint32_t)(t->Hp * t->Wp)), p.drow = make_fastdiv((uint32_t)t->Wp);
    p.out = out, p.bias = bias, p.acc = acc, p.status = d->status;
    p.splits = 1;
    CUtensorMap m[4];
    bool ok;
    int64_t qlen, qrows;  // Q matrix: qrows rows of qlen floats
    if (mode == MODE_FWD) {
        p.R = Nv, p.Cq = g->OC, p.CB = (int)(Cp / 32), p.sgn = 1;
        p.eh = 0, p.ew = 0, p.DH = (int)g->OH, p.DW = (int)g->OW;
        p.out_img = g->OC * g->OH * g->OW, p.out_ch = g->OH * g->OW;
        qlen = T * Cp, qrows = g->OC;
    } else if (mode == MODE_DX) {
        p.R = Nv, p.Cq = g->C, p.CB = (int)(OCp / 32), p.sgn = -1;
        p.eh = g->ph, p.ew = g->pw, p.DH = (int)g->H, p.DW = (int)g->W;
        p.out_img = g->C * g->H * g->W, p.out_ch = g->H * g->W;
        qlen = T * OCp, qrows = g->C;
    } else {
        p.R = T * Cp, p.Cq = g->OC, p.CB = (int)(Cp / 32), p.sgn = 1, p.K = Nv;
        qlen = OCp, qrows = Nv;
    }
    p.ksteps = (int)(T * p.CB);
    p.BN = ct_pick_bn(p.Cq);
    const int64_t plen = mode == MODE_DX ? OCp : Cp;  // P: Nv rows of plen floats
    if (mode != MODE_DW) {
        ok = make_map(&m[0], P, plen, Nv, plen, 1, 0, TK, TM, false) &&
             make_map(&m[2], Q, qlen, qrows, qlen, 1, 0, TK, p.BN, false);
        if (three)
            ok = ok && make_map(&m[1], P + Nv * plen, plen, Nv, plen, 1, 0, TK, TM, false) &&
                 make_map(&m[3], Q + qrows * qlen, qlen, qrows, qlen, 1, 0, TK, p.BN, false);
    } else {
        ok = make_map(&m[0], P, plen, Nv, plen, 1, 0, 32, TK, true) &&
             make_map(&m[2], Q, qlen, qrows, qlen, 1, 0, 32, TK, true);
        if (three)
            ok = ok && make_map(&m[1], P + Nv * plen, plen, Nv, plen, 1, 0, 32, TK, true) &&
                 make_map(&m[3], Q + qrows * qlen, qlen, qrows, qlen, 1, 0, 32, TK, true);
    }
    if (!ok) return 0;
    if (!three) m[1] = m[0], m[3] = m[2];

    p.tiles_r = (p.R + TM - 1) / TM, p.tiles_q = (p.Cq + p.BN - 1) / p.BN;
    const int64_t tiles = p.tiles_r * p.tiles_q, sms = d->sm_count > 0 ? d->sm_count : 148;
    if (mode == MODE_DW) {
        // the sum over positions is split into slices so that every SM has work; each slice writes a
        // partial tile and the combine kernel adds the slices in a fixed order
        // at most one unit per SM: a unit more than the grid would run as a second wave on its own
        int64_t splits = sms / tiles > 1 ? sms / tiles : 1;
        const int64_t cap_k = (Nv + 8 * TK - 1) / (8 * TK);  // at least 8 K steps per slice
        const int64_t cap_mem = (int64_t)(d->scratch_bytes / sizeof(float)) / (p.R * p.Cq);
        if (splits > cap_k) splits = cap_k;
        if (splits > cap_mem) splits = cap_mem;
        if (splits < 1) return 0;
        p.kper = ((Nv + splits - 1) / splits + TK - 1) / TK * TK;
        splits = (Nv + p.kper - 1) / p.kper;
        p.splits = (int)splits;
        p.part = (float *)d->scratch;
    }
    p.units = tiles * p.splits;
    const size_t per = (size_t)(kStageA + p.BN * TK) * 4 * (three ? 2 : 1);
    size_t nst = (kSmemLimit - 2048) / per;
    p.stages = (int)(nst > (size_t)kMaxStages ? kMaxStages : nst);
    const size_t smem = 2048 + (size_t)p.stages * per;
    const unsigned grid = (unsigned)(p.units < sms ? p.units : sms);

    static const char *names[3] = {"conv_tap_fwd", "conv_tap_dx", "conv_tap_dw"};
    const double flops = 2.0 * g->N * g->OC * g->C * T * g->OH * g->OW;
    const double pl = (double)t->planes;
    double bytes;
    if (mode == MODE_FWD) bytes = 4.0 * (pl * (Nv * Cp + qrows * qlen) + (double)g->N * g->OC * g->OH * g->OW);
    else if (mode == MODE_DX) bytes = 4.0 * (pl * (Nv * OCp + qrows * qlen) + (acc ? 2.0 : 1.0) * g->N * g->C * g->H * g->W);
    else bytes = 4.0 * (pl * Nv * (Cp + OCp) + 2.0 * g->OC * g->C * T);
    Scope sc(d, names[mode], flops, bytes);
    bool launched = mode == MODE_FWD ? ct_launch<MODE_FWD>(d, three, grid, smem, m, p)
                    : mode == MODE_DX ? ct_launch<MODE_DX>(d, three, grid, smem, m, p)
                                      : ct_launch<MODE_DW>(d, three, grid, smem, m, p);
    if (!launched) return 0;
    if (cudaGetLastError() != cudaSuccess) {
        *(volatile int *)d->status_host = NCK_ERR_LAUNCH;
        return 1;
    }
    int n = 1;
    if (mode == MODE_DW) {
        k_tap_dw_combine<<<grid_for(d, g->OC * g->C * T), kThreads, 0, NCK_STREAM(d)>>>(
            p.part, out, p.splits, p.R, p.Cq, (int)g->C, (int)T, (int)Cp, acc);
        n++;
    }
    NCK_LAUNCHED(d, n);
    return 1;
}
