// FP32-input GEMM on the 5th-generation tensor cores: tcgen05.mma kind::tf32, operands staged in
// shared memory by TMA (128-byte swizzle, no multicast), accumulators in tensor memory.
//
// Orientation. The kernel computes D[i][j] = sum_k P[i][k] * Q[j][k] with the 128 rows i of a tile
// on the 128 TMEM lanes, and stores D[i][j] at out[j * ldo + i]. The host passes P = op(B)^T and
// Q = op(A), so i runs along C's contiguous dimension (n) and every warp store of the epilogue
// writes 32 consecutive floats. The tile width BN (Q rows per tile) is chosen per GEMM among
// 32, 64, 96, 128 to fit M (64 output channels use a 64-wide tile, 288 a 96-wide one).
//
// Persistent CTAs, one per SM, walk a static list of work units (tile, output batch, reduction slice)
// with warp-specialised roles:
//   warps 0-3  epilogue: tcgen05.ld of the accumulator rows (warp w owns lanes 32w..32w+31), alpha /
//              bias / beta, coalesced stores (or raw partial tiles when the reduction is split)
//   warp 4     TMA loader (one thread) feeding a ring of up to 8 stages, K in steps of 32 (128 B)
//   warp 5     MMA issuer (one thread): 4 MMAs of K = 8 per stage, commits each stage back to the
//              loader and each finished tile to the epilogue
//   warps 6-13 3xTF32 only: write the remainder of every staged fp32 tile below its TF32 head (the
//              top 19 bits, which the MMA reads from the staged tile itself), rounded to TF32; the Q
//              remainder lands right after the Q head, so the MMA thread issues two MMAs per K step:
//              P_head x [Q_head | Q_rest] into a 2*BN-wide accumulator, then P_rest x Q_head into its
//              first half; the epilogue adds the halves
// Two accumulators in TMEM let the epilogue of one tile overlap the main loop of the next.
//
// Every mbarrier wait gives up after 2 s of device time and records an error in the status word; a
// role that gave up stops, the loader waits (bounded) for its copies in flight, the MMA thread for
// its MMAs, and the CTA frees its TMEM and returns.
#include <cuda.h>
#include <string.h>

#include "k_common.cuh"
#include "k_tcgen05.cuh"

using namespace nck;

namespace {

using namespace tc;

constexpr int kEpiWarps = 4, kLoadWarp = 4, kMmaWarp = 5, kSplitWarp0 = 6, kSplitThreads = 256;
constexpr int kThreadsTf32 = kSplitWarp0 * 32, kThreads3x = kThreadsTf32 + kSplitThreads;

struct TcParams {
    int64_t R, Cq, K;      // P rows (original N), Q rows (original M), depth
    int BN;                // tile width along Q
    int stages;            // ring depth (as many as shared memory holds, at most kMaxStages)
    float alpha, beta;
    float *C;
    int64_t ldc, sC;
    const float *bias;
    int bias_q;            // bias indexed by the Q row (original row m); else by the P row (column n)
    int64_t batch;
    int reduce, splits;    // reduce: the batch is summed; splits: slices of the reduction range
    int64_t bper, kper;    // batches per slice (reduce), K per slice (otherwise)
    int64_t tiles_r, tiles_q, units;
    float *part;           // partial tiles [unit slice][Cq][R] when splits > 1
    int p_mn, q_mn;        // operand stored MN-major
    int p_bat, q_bat;      // operand has a batch coordinate (3-D tensor map)
    int *status;
};

// Barriers sit in the first KiB of dynamic shared memory; the stage buffers follow, 1 KiB aligned:
// [P stages][Q stages] and in 3xTF32 mode [P rests]; in 3xTF32 mode a Q stage holds the head tile
// followed by its remainder (2 * BN rows).
struct Bars {
    uint64_t full[kMaxStages], empty[kMaxStages], ready[kMaxStages];
    uint64_t tfull[2], tempty[2], mma_done;
    uint32_t tmem;
};

// A work unit: tile (tr, tq), output batch ob (or 0 when the batch is summed), reduction slice sl.
struct Unit {
    int64_t r0, q0, ob, sl, b0, b1, k0, k1, steps;
};

__device__ __forceinline__ Unit unit_of(const TcParams &p, int64_t u) {
    Unit w;
    int64_t tiles = p.tiles_r * p.tiles_q;
    int64_t t = u % tiles, z = u / tiles;
    w.r0 = (t % p.tiles_r) * TM;
    w.q0 = (t / p.tiles_r) * p.BN;
    if (p.reduce) {
        w.ob = 0, w.sl = z;
        w.b0 = z * p.bper;
        w.b1 = w.b0 + p.bper < p.batch ? w.b0 + p.bper : p.batch;
        w.k0 = 0, w.k1 = p.K;
    } else {
        w.ob = z / p.splits, w.sl = z % p.splits;
        w.b0 = w.ob, w.b1 = w.ob + 1;
        w.k0 = w.sl * p.kper;
        w.k1 = w.k0 + p.kper < p.K ? w.k0 + p.kper : p.K;
    }
    int64_t kt = (w.k1 - w.k0 + TK - 1) / TK;
    w.steps = (w.b1 - w.b0) * kt;
    return w;
}

// 3xTF32: the accumulator's second half (P_h Q_r) added to the first (P_h Q_h + P_r Q_h), column by column
__device__ __forceinline__ void add_cross(uint32_t taddr, uint32_t (&r)[16]) {
    uint32_t r2[16];
    tmem_ld16(taddr, r2);
#pragma unroll
    for (int j = 0; j < 16; j++) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(r2[j]));
}

template <bool THREE, bool BETA>
__global__ void __launch_bounds__(THREE ? kThreads3x : kThreadsTf32, 1) k_tcgemm(const __grid_constant__ CUtensorMap tmP,
                                                                 const __grid_constant__ CUtensorMap tmQ, TcParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~(uintptr_t)1023);
    Bars &s = *reinterpret_cast<Bars *>(base);
    const int S = p.stages, sbq = p.BN * TK, sbq2 = THREE ? 2 * sbq : sbq;
    float *const ring_a = reinterpret_cast<float *>(base + 1024);
    float *const ring_b = ring_a + S * kStageA;
    float *const rest_a = ring_b + S * sbq2;  // 3xTF32 only
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int BN = p.BN;
    const int AW = THREE ? 2 * BN : BN;  // accumulator columns per tile
    const uint32_t tcols = tmem_cols(AW);
    const uint32_t stage_bytes = (uint32_t)(TM + BN) * TK * 4;

    if (tid == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
            mbar_init(&s.ready[i], kSplitThreads);
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
            // stage, phase, batch and K position advance by counting: no division per K step
            int64_t it = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                Unit w = unit_of(p, u);
                int b = (int)w.b0, kk = (int)w.k0;
                for (int64_t t = 0; t < w.steps; t++, it++) {
                    if (it >= S && !(ok = mbar_wait(&s.empty[st], ph ^ 1, p.status))) break;
                    mbar_expect_tx(&s.full[st], stage_bytes);
                    if (!p.p_mn) {
                        if (p.p_bat) tma_3d(ring_a + st * kStageA, &tmP, kk, (int)w.r0, b, &s.full[st]);
                        else tma_2d(ring_a + st * kStageA, &tmP, kk, (int)w.r0, &s.full[st]);
                    } else {
                        for (int j = 0; j < TM / 32; j++) {
                            if (p.p_bat) tma_3d(ring_a + st * kStageA + j * 1024, &tmP, (int)w.r0 + 32 * j, kk, b, &s.full[st]);
                            else tma_2d(ring_a + st * kStageA + j * 1024, &tmP, (int)w.r0 + 32 * j, kk, &s.full[st]);
                        }
                    }
                    if (!p.q_mn) {
                        if (p.q_bat) tma_3d(ring_b + st * sbq2, &tmQ, kk, (int)w.q0, b, &s.full[st]);
                        else tma_2d(ring_b + st * sbq2, &tmQ, kk, (int)w.q0, &s.full[st]);
                    } else {
                        for (int j = 0; j < BN / 32; j++) {
                            if (p.q_bat) tma_3d(ring_b + st * sbq2 + j * 1024, &tmQ, (int)w.q0 + 32 * j, kk, b, &s.full[st]);
                            else tma_2d(ring_b + st * sbq2 + j * 1024, &tmQ, (int)w.q0 + 32 * j, kk, &s.full[st]);
                        }
                    }
                    if (++st == S) st = 0, ph ^= 1;
                    kk += TK;
                    if (kk >= w.k1) kk = (int)w.k0, b++;
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
            const uint32_t idesc = idesc_tf32(p.p_mn, p.q_mn, BN), idesc2 = idesc_tf32(p.p_mn, p.q_mn, 2 * BN);
            const uint64_t dA = stage_desc(smem_u32(ring_a), p.p_mn, 0), dB = stage_desc(smem_u32(ring_b), p.q_mn, 0);
            const uint32_t stA = (uint32_t)(kStageA * 4) >> 4, stB = (uint32_t)(sbq2 * 4) >> 4;
            const uint32_t kA = p.p_mn ? 64u : 2u, kB = p.q_mn ? 64u : 2u;  // 8 K rows (MN-major) or 32 B
            const uint64_t restA = (uint64_t)((smem_u32(rest_a) - smem_u32(ring_a)) >> 4);
            int64_t it = 0, local = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, local++) {
                Unit w = unit_of(p, u);
                int acc = (int)(local & 1);
                if (local >= 2 && !(ok = mbar_wait(&s.tempty[acc], (uint32_t)(((local >> 1) & 1) ^ 1), p.status)))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + (uint32_t)acc * (tcols / 2);
                for (int64_t t = 0; t < w.steps; t++, it++) {
                    if (!(ok = mbar_wait(THREE ? &s.ready[st] : &s.full[st], ph, p.status))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    // descriptors by addition: the start address (bits 0-13, in 16-byte units) is the only
                    // field that moves between stages and K steps
                    const uint64_t a0 = dA + (uint64_t)(st * stA), b0 = dB + (uint64_t)(st * stB);
#pragma unroll
                    for (int k = 0; k < TK / 8; k++) {
                        const uint32_t accum = (t > 0 || k > 0) ? 1u : 0u;
                        const uint64_t ak = a0 + (uint64_t)(k * kA), bk = b0 + (uint64_t)(k * kB);
                        if (THREE) {
                            mma_tf32(d, ak, bk, idesc2, accum);     // [P_h Q_h | P_h Q_r]
                            mma_tf32(d, ak + restA, bk, idesc, 1u);  // += P_r Q_h in the first half
                        } else {
                            mma_tf32(d, ak, bk, idesc, accum);
                        }
                    }
                    mma_commit(&s.empty[st]);  // the loader may refill this stage once these MMAs read it
                    if (++st == S) st = 0, ph ^= 1;
                }
                if (ok) mma_commit(&s.tfull[acc]);
            }
            // every MMA issued has completed before the CTA frees tensor memory
            mma_commit(&s.mma_done);
            mbar_wait(&s.mma_done, 0, p.status);
        }
    } else if (THREE && warp >= kSplitWarp0) {
        // ---- 3xTF32 split: head = x with the low 13 mantissa bits cleared, rest = x - head rounded to
        // the nearest TF32 value. The tensor core reads an fp32 operand as TF32 by dropping those 13 bits
        // (truncation, checked on B200), so the staged x already serves as the head and only the rest is
        // written --------------------------------------------------------------------------------------
        const int t2 = tid - kSplitWarp0 * 32;  // 0 .. kSplitThreads - 1
        const int nb = BN * TK / 4;
        int st = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
            Unit w = unit_of(p, u);
            for (int64_t t = 0; t < w.steps; t++) {
                if (!(ok = mbar_wait(&s.full[st], ph, p.status))) break;
                float4 *ah = reinterpret_cast<float4 *>(ring_a + st * kStageA), *al = reinterpret_cast<float4 *>(rest_a + st * kStageA);
                for (int i = t2; i < TM * TK / 4; i += kSplitThreads) {
                    al[i] = tf32_rest4(ah[i]);
                }
                float4 *bh = reinterpret_cast<float4 *>(ring_b + st * sbq2), *bl = bh + sbq / 4;
                for (int i = t2; i < nb; i += kSplitThreads) {
                    bl[i] = tf32_rest4(bh[i]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
                mbar_arrive(&s.ready[st]);
                if (++st == S) st = 0, ph ^= 1;
            }
        }
    } else if (warp < kEpiWarps) {
        // ---- epilogue: accumulator lane i = P row r0 + 32 * warp + lane ---------------------------------
        int64_t local = 0;
        const bool partial = p.splits > 1;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x, local++) {
            Unit w = unit_of(p, u);
            int acc = (int)(local & 1);
            if (!mbar_wait(&s.tfull[acc], (uint32_t)((local >> 1) & 1), p.status)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int64_t i = w.r0 + warp * 32 + lane;
            // partial tiles: slice-major [ob][slice][Cq][R] (ob = 0 when the batch is summed)
            float *out = partial ? p.part + (w.ob * p.splits + w.sl) * p.R * p.Cq : p.C + w.ob * p.sC;
            const int64_t ldo = partial ? p.R : p.ldc;
            const bool live = i < p.R;
            const float bias_i = (!partial && p.bias && !p.bias_q && live) ? p.bias[i] : 0.0f;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)acc * (tcols / 2) + (uint32_t)c0;
                if (BETA && !partial) {
                    // C is fetched before the accumulator read, all 16 loads in flight at once
                    float cv[16];
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) {
                        const int64_t j = w.q0 + c0 + jj;
                        cv[jj] = (live && j < p.Cq) ? out[j * ldo + i] : 0.0f;
                    }
                    tmem_ld16(taddr, r);
                    if (THREE) add_cross(taddr + (uint32_t)BN, r);
                    if (!live) continue;
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) {
                        const int64_t j = w.q0 + c0 + jj;
                        if (j < p.Cq) {
                            float v = p.alpha * __uint_as_float(r[jj]);
                            if (p.bias) v = v + (p.bias_q ? p.bias[j] : bias_i);
                            out[j * ldo + i] = fmaf(p.beta, cv[jj], v);
                        }
                    }
                    continue;
                }
                tmem_ld16(taddr, r);
                if (THREE) add_cross(taddr + (uint32_t)BN, r);
                if (!live) continue;
#pragma unroll
                for (int jj = 0; jj < 16; jj++) {
                    int64_t j = w.q0 + c0 + jj;
                    if (j >= p.Cq) break;
                    float a = __uint_as_float(r[jj]);
                    float *dst = out + j * ldo + i;
                    if (partial) {
                        *dst = a;
                    } else {
                        float v = p.alpha * a;
                        if (p.bias) v = v + (p.bias_q ? p.bias[j] : bias_i);
                        *dst = v;
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

// C = alpha * (sum of the slices' partial tiles) + bias + beta * C, slices added in a fixed order
__global__ void k_tc_combine(TcParams p, int64_t nout) {
    int64_t MN = p.R * p.Cq, total = nout * MN;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ob = t / MN, r = t - ob * MN, m = r / p.R, n = r - m * p.R;
        const float *src = p.part + ob * p.splits * MN + r;
        // slices in order over four interleaved running sums (k mod 4), added at the end
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        int k = 0;
        for (; k + 4 <= p.splits; k += 4)
            s0 += __ldcg(src + k * MN), s1 += __ldcg(src + (k + 1) * MN), s2 += __ldcg(src + (k + 2) * MN),
                s3 += __ldcg(src + (k + 3) * MN);
        for (; k < p.splits; k++) s0 += __ldcg(src + k * MN);
        const float s = (s0 + s1) + (s2 + s3);
        float *c = p.C + ob * p.sC + m * p.ldc + n;
        float v = p.alpha * s;
        if (p.bias) v = v + (p.bias_q ? p.bias[m] : p.bias[n]);
        if (p.beta != 0.0f) v = fmaf(p.beta, *c, v);
        *c = v;
    }
}

// ---- host side -------------------------------------------------------------------------------------

// stages that fit: per stage a P tile (16 KiB) and a Q tile (BN * 128 B), doubled in 3xTF32 mode
int ring_stages(int bn, bool three) {
    size_t per = (size_t)(kStageA + bn * TK) * 4 * (three ? 2 : 1);
    size_t n = (kSmemLimit - 2048) / per;
    return (int)(n > (size_t)kMaxStages ? kMaxStages : n);
}

size_t smem_bytes(int bn, bool three, int stages) {
    return 2048 + (size_t)stages * (kStageA + bn * TK) * 4 * (three ? 2 : 1);
}

// tile width along Q: the fewest wasted columns, counting ~32 columns of per-tile overhead
int pick_bn(int64_t cq) {
    int best = 128;
    int64_t best_cost = INT64_MAX;
    for (int bn = 32; bn <= kMaxBN; bn += 32) {
        int64_t tiles = (cq + bn - 1) / bn, cost = tiles * (bn + 32);
        if (cost < best_cost) best_cost = cost, best = bn;
    }
    return best;
}

template <bool THREE, bool BETA>
bool set_smem_attr() {
    static int done = 0;
    if (done) return true;
    if (cudaFuncSetAttribute(k_tcgemm<THREE, BETA>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    done = 1;
    return true;
}

}  // namespace

// Returns 1 when the GEMM was launched on the tensor cores, 0 when its layout does not fit the TMA
// constraints (16-byte aligned bases and strides) and the caller should use the FFMA kernel.
extern "C" int nck_gemm_tc(nck_dev *d, const nck_gemm_args *a) {
    if (a->M <= 0 || a->N <= 0 || a->batch <= 0 || a->K <= 0) return 0;
    if (a->M > INT32_MAX || a->N > INT32_MAX || a->K > INT32_MAX || a->batch > INT32_MAX) return 0;
    const int three = d->gemm_mode == NCK_GEMM_3XTF32;
    // P = op(B)^T (rows n), Q = op(A) (rows m)
    const int p_mn = !a->tb, q_mn = a->ta;
    const int p_bat = a->batch > 1 && a->sB != 0, q_bat = a->batch > 1 && a->sA != 0;
    if ((uintptr_t)a->A % 16 || (uintptr_t)a->B % 16 || a->lda % 4 || a->ldb % 4) return 0;
    if ((p_bat && a->sB % 4) || (q_bat && a->sA % 4)) return 0;
    const int bn = pick_bn(a->M);
    CUtensorMap mp, mq;
    bool okP = !p_mn ? make_map(&mp, a->B, a->K, a->N, a->ldb, p_bat ? a->batch : 1, a->sB, TK, TM, false)
                     : make_map(&mp, a->B, a->N, a->K, a->ldb, p_bat ? a->batch : 1, a->sB, 32, TK, true);
    bool okQ = !q_mn ? make_map(&mq, a->A, a->K, a->M, a->lda, q_bat ? a->batch : 1, a->sA, TK, bn, false)
                     : make_map(&mq, a->A, a->M, a->K, a->lda, q_bat ? a->batch : 1, a->sA, 32, TK, true);
    if (!okP || !okQ) return 0;

    TcParams p;
    memset(&p, 0, sizeof p);
    p.R = a->N, p.Cq = a->M, p.K = a->K, p.BN = bn, p.alpha = a->alpha, p.beta = a->beta;
    p.C = a->C, p.ldc = a->ldc, p.sC = a->sC, p.bias = a->bias, p.bias_q = a->bias_per_row;
    p.batch = a->batch, p.reduce = a->reduce_batch && a->batch > 1;
    p.p_mn = p_mn, p.q_mn = q_mn, p.p_bat = p_bat, p.q_bat = q_bat, p.status = d->status;
    p.tiles_r = (a->N + TM - 1) / TM, p.tiles_q = (a->M + bn - 1) / bn;

    const int64_t tiles = p.tiles_r * p.tiles_q, nout = p.reduce ? 1 : a->batch;
    const int64_t sms = d->sm_count > 0 ? d->sm_count : 148;
    const int64_t maxpart = (int64_t)(d->scratch_bytes / sizeof(float)) / (a->M * a->N * nout);
    int64_t splits = 1;
    if (p.reduce) {
        // the batch sum: a slice per SM (no more units than SMs), each slice a run of whole samples
        splits = sms / tiles > 1 ? sms / tiles : 1;
        if (splits > a->batch) splits = a->batch;
    } else if (tiles * nout < sms) {
        // no more units than SMs: one unit over the grid would run as a second wave on its own
        splits = sms / (tiles * nout);
        int64_t cap = (a->K + 4 * TK - 1) / (4 * TK);
        if (splits > cap) splits = cap;
    }
    if (splits > maxpart) splits = maxpart;
    if (splits < 1) splits = 1;
    if (p.reduce) {
        p.bper = (a->batch + splits - 1) / splits;
        splits = (a->batch + p.bper - 1) / p.bper;
        p.kper = a->K;
    } else {
        p.bper = 1;
        p.kper = ((a->K + splits - 1) / splits + TK - 1) / TK * TK;
        splits = (a->K + p.kper - 1) / p.kper;
    }
    p.splits = (int)splits;
    p.part = (float *)d->scratch;
    p.units = tiles * nout * splits;

    const bool beta = a->beta != 0.0f;
    const bool attr = three ? (beta ? set_smem_attr<true, true>() : set_smem_attr<true, false>())
                            : (beta ? set_smem_attr<false, true>() : set_smem_attr<false, false>());
    if (!attr) return 0;
    p.stages = ring_stages(bn, three);
    const size_t smem = smem_bytes(bn, three, p.stages);
    const double nA = a->sA ? (double)a->batch : 1.0, nB = a->sB ? (double)a->batch : 1.0;
    const double nC = (double)nout * (a->beta != 0.0f ? 2.0 : 1.0);
    Scope sc(d, three ? "gemm_3xtf32_tc" : "gemm_tf32_tc", 2.0 * a->M * a->N * a->K * a->batch,
             4.0 * (nA * a->M * a->K + nB * a->K * a->N + nC * a->M * a->N));
    const unsigned grid = (unsigned)(p.units < sms ? p.units : sms);
    if (three && beta) k_tcgemm<true, true><<<grid, kThreads3x, smem, NCK_STREAM(d)>>>(mp, mq, p);
    else if (three) k_tcgemm<true, false><<<grid, kThreads3x, smem, NCK_STREAM(d)>>>(mp, mq, p);
    else if (beta) k_tcgemm<false, true><<<grid, kThreadsTf32, smem, NCK_STREAM(d)>>>(mp, mq, p);
    else k_tcgemm<false, false><<<grid, kThreadsTf32, smem, NCK_STREAM(d)>>>(mp, mq, p);
    if (cudaGetLastError() != cudaSuccess) {
        /* a launch that never ran: report it through the status word like a kernel-found error */
        *(volatile int *)d->status_host = NCK_ERR_LAUNCH;
        return 1;
    }
    int launched = 1;
    if (splits > 1) {
        k_tc_combine<<<grid_for(d, nout * a->M * a->N), kThreads, 0, NCK_STREAM(d)>>>(p, nout);
        launched++;
    }
    NCK_LAUNCHED(d, launched);
    return 1;
}

// A pipeline wait that nothing completes: an mbarrier expecting one arrival that never comes. The
// bounded wait gives up after kWaitNs and reports kErrPipeline, the path every tcgen05 kernel takes
// when a TMA transfer or an MMA commit does not arrive; it exercises that reporting end to end.
__global__ void k_wait_probe(int *status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, status);
}

extern "C" void nck_pipeline_wait_probe(nck_dev *d) {
    k_wait_probe<<<1, 32, 0, NCK_STREAM(d)>>>(d->status);
    NCK_LAUNCHED(d, 1);
}
