// FP32-input GEMM on the 5th-generation tensor cores: tcgen05.mma kind::tf32, operands staged in
// shared memory by TMA (128-byte swizzle, no multicast), accumulator in tensor memory, one CTA per
// 128 x 128 output tile.
//
// Roles in a 128-thread CTA: thread 0 issues the TMA loads of a 4-stage ring (3 in 3xTF32 mode), thread 32 issues the
// MMAs (4 x K=8 per 32-deep stage) and commits each stage back to the loader, then all four warps
// read the accumulator rows out of TMEM (warp w owns lanes 32w .. 32w+31 = tile rows) and apply the
// epilogue C = alpha * acc + bias + beta * C, or store raw partial tiles when the reduction range is
// split. In 3xTF32 mode two more warps split every staged fp32 tile into a TF32-exact high part and
// the remainder, and the MMA thread accumulates hi*hi + hi*lo + lo*hi: close to fp32 accuracy.
//
// Every wait on an mbarrier gives up after 2 s of device time and records an error in the context's
// status word, so a broken pipeline cannot hang the GPU.
#include <cuda.h>
#include <string.h>

#include "k_common.cuh"

using namespace nck;


namespace {

constexpr int TM = 128, TN = 128, TK = 32;  // tile; TK fp32 = 128 bytes = one swizzle row
constexpr int kTileBytes = TM * TK * 4;      // 16 KiB per operand per stage
constexpr uint64_t kWaitNs = 2000000000ull;   // an mbarrier wait gives up after 2 s of device time
constexpr int kErrPipeline = 3;              // status code for a wait that gave up

struct TcParams {
    int64_t M, N, K;
    float alpha, beta;
    float *C;
    int64_t ldc, sC;
    const float *bias;
    int bias_row;
    int64_t batch;
    int reduce, splits;
    int64_t bper, kper;
    float *part;
    int a_mn, b_mn;      // operand stored MN-major (transposed relative to K-major)
    int a_bat, b_bat;    // operand has a batch coordinate (3-D tensor map)
    int three;           // 3xTF32
    int *status;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// returns false when the bounded wait gave up (the error goes to the status word)
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status) {
    uint32_t addr = smem_u32(bar);
    uint64_t start = 0;
    for (uint32_t i = 0;; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred P;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, P;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 1023) == 0) {
            uint64_t t = now_ns();
            if (!start) start = t;
            else if (t - start > kWaitNs) break;
        }
    }
    report(status, kErrPipeline);
    return false;
}

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// shared memory matrix descriptor, version 1 (sm100); layout 2 = 128-byte swizzle in 16-byte units
// (K-major tiles), layout 1 = 128-byte swizzle in 32-byte units (the only MN-major form for tf32)
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // version
    d |= (uint64_t)layout << 61;
    return d;
}

// instruction descriptor: D f32, A/B tf32, dense, M = 128, N = 128
__device__ __forceinline__ uint32_t idesc_tf32(int a_mn, int b_mn) {
    uint32_t d = 0;
    d |= 1u << 4;               // D format F32
    d |= 2u << 7;               // A format TF32
    d |= 2u << 10;              // B format TF32
    d |= (uint32_t)a_mn << 15;  // A major
    d |= (uint32_t)b_mn << 16;  // B major
    d |= (uint32_t)(TN >> 3) << 17;
    d |= (uint32_t)(TM >> 4) << 24;
    return d;
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// K-offset descriptors of one stage buffer for the k-th 8-deep MMA step
__device__ __forceinline__ uint64_t stage_desc(uint32_t base, int mn, int k) {
    // K-major: 128 B rows of 32 K values, 8-row atoms 1024 B apart; step k moves 32 B along the row
    if (!mn) return sdesc(base + k * 32, 16, 1024, 2);
    // MN-major: 128 B rows of 32 M/N values, one row per K; 4-row atoms 512 B apart (SBO), 32-wide
    // blocks 4 KiB apart (LBO); step k moves 8 rows
    return sdesc(base + k * 1024, 4096, 512, 1);
}

template <int S>
struct Smem {
    float a[S][TM * TK];
    float b[S][TN * TK];
    uint64_t full[S], empty[S], ready[S], lo_free[S], accum;
    uint32_t tmem;
};

template <int S>
struct SmemLo {
    float a[S][TM * TK];
    float b[S][TN * TK];
};

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// S pipeline stages; THREE selects 3xTF32 (two extra warps split the staged tiles)
template <int S, bool THREE>
__global__ void __launch_bounds__(THREE ? 192 : 128, 1) k_tcgemm(const __grid_constant__ CUtensorMap tmA,
                                                                 const __grid_constant__ CUtensorMap tmB, TcParams p) {
    constexpr int kStages = S;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment of the stage buffers (the swizzle pattern follows address bits)
    Smem<S> &s = *reinterpret_cast<Smem<S> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    SmemLo<S> *lo = THREE ? reinterpret_cast<SmemLo<S> *>(reinterpret_cast<unsigned char *>(&s) +
                                                          ((sizeof(Smem<S>) + 1023) & ~(size_t)1023))
                          : nullptr;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n0 = (int64_t)blockIdx.x * TN, m0 = (int64_t)blockIdx.y * TM, z = blockIdx.z;

    int64_t b0, b1, k0 = 0, k1 = p.K, ob;
    if (p.reduce) {
        b0 = z * p.bper;
        b1 = b0 + p.bper < p.batch ? b0 + p.bper : p.batch;
        ob = 0;
    } else {
        ob = z / p.splits;
        int64_t sl = z % p.splits;
        b0 = ob, b1 = ob + 1;
        k0 = sl * p.kper;
        k1 = k0 + p.kper < p.K ? k0 + p.kper : p.K;
    }
    const int64_t kt_n = (k1 - k0 + TK - 1) / TK;
    const int64_t T = (b1 > b0 ? b1 - b0 : 0) * kt_n;

    if (tid == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
            mbar_init(&s.ready[i], 64);   // the two split warps (3xTF32)
            mbar_init(&s.lo_free[i], 1);
        }
        mbar_init(&s.accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(TN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;
    bool ok = true;
    if (tid == 0) {
    }

    if (tid == 0) {
        // ---- loader --------------------------------------------------------------------------
        for (int64_t t = 0; t < T && ok; t++) {
            int st = (int)(t % kStages);
            uint32_t ph = (uint32_t)((t / kStages) & 1);
            if (t >= kStages) ok = mbar_wait(&s.empty[st], ph ^ 1, p.status);
            if (!ok) break;
            int64_t b = b0 + t / kt_n;
            int kk = (int)(k0 + (t % kt_n) * TK);
            mbar_expect_tx(&s.full[st], 2 * kTileBytes);
            if (!p.a_mn) {
                if (p.a_bat) tma_3d(s.a[st], &tmA, kk, (int)m0, (int)b, &s.full[st]);
                else tma_2d(s.a[st], &tmA, kk, (int)m0, &s.full[st]);
            } else {
                for (int j = 0; j < 4; j++) {
                    if (p.a_bat) tma_3d(s.a[st] + j * 1024, &tmA, (int)m0 + 32 * j, kk, (int)b, &s.full[st]);
                    else tma_2d(s.a[st] + j * 1024, &tmA, (int)m0 + 32 * j, kk, &s.full[st]);
                }
            }
            if (!p.b_mn) {
                if (p.b_bat) tma_3d(s.b[st], &tmB, kk, (int)n0, (int)b, &s.full[st]);
                else tma_2d(s.b[st], &tmB, kk, (int)n0, &s.full[st]);
            } else {
                for (int j = 0; j < 4; j++) {
                    if (p.b_bat) tma_3d(s.b[st] + j * 1024, &tmB, (int)n0 + 32 * j, kk, (int)b, &s.full[st]);
                    else tma_2d(s.b[st] + j * 1024, &tmB, (int)n0 + 32 * j, kk, &s.full[st]);
                }
            }
        }
    } else if (tid == 32) {
        // ---- MMA issuer -------------------------------------------------------------------------
        const uint32_t idesc = idesc_tf32(p.a_mn, p.b_mn);
        for (int64_t t = 0; t < T && ok; t++) {
            int st = (int)(t % kStages);
            uint32_t ph = (uint32_t)((t / kStages) & 1);
            ok = mbar_wait(THREE ? &s.ready[st] : &s.full[st], ph, p.status);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            uint32_t ab = smem_u32(s.a[st]), bb = smem_u32(s.b[st]);
            for (int k = 0; k < TK / 8; k++) {
                uint32_t acc = (t > 0 || k > 0) ? 1u : 0u;
                mma_tf32(tmem, stage_desc(ab, p.a_mn, k), stage_desc(bb, p.b_mn, k), idesc, acc);
                if (THREE) {
                    uint32_t al = smem_u32(lo->a[st]), bl = smem_u32(lo->b[st]);
                    mma_tf32(tmem, stage_desc(ab, p.a_mn, k), stage_desc(bl, p.b_mn, k), idesc, 1u);
                    mma_tf32(tmem, stage_desc(al, p.a_mn, k), stage_desc(bb, p.b_mn, k), idesc, 1u);
                }
            }
            mma_commit(&s.empty[st]);  // the loader may refill this stage once these MMAs have read it
            if (THREE) mma_commit(&s.lo_free[st]);
        }
        mma_commit(&s.accum);
    } else if (THREE && warp >= 4) {
        // ---- 3xTF32 split: hi = x with the low 13 mantissa bits cleared, lo = x - hi --------------
        const int t2 = tid - 128;  // 0 .. 63
        for (int64_t t = 0; t < T && ok; t++) {
            int st = (int)(t % kStages);
            uint32_t ph = (uint32_t)((t / kStages) & 1);
            ok = mbar_wait(&s.full[st], ph, p.status);
            if (ok && t >= kStages) ok = mbar_wait(&s.lo_free[st], ph ^ 1, p.status);
            if (!ok) break;
            float4 *ah = reinterpret_cast<float4 *>(s.a[st]), *bh = reinterpret_cast<float4 *>(s.b[st]);
            float4 *al = reinterpret_cast<float4 *>(lo->a[st]), *bl = reinterpret_cast<float4 *>(lo->b[st]);
            for (int i = t2; i < TM * TK / 4; i += 64) {
                float4 v = ah[i], h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                ah[i] = h;
                al[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
                float4 u = bh[i], g = make_float4(tf32_hi(u.x), tf32_hi(u.y), tf32_hi(u.z), tf32_hi(u.w));
                bh[i] = g;
                bl[i] = make_float4(u.x - g.x, u.y - g.y, u.z - g.z, u.w - g.w);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
            mbar_arrive(&s.ready[st]);
        }
    }

    // ---- epilogue: warps 0-3, row m0 + 32 * warp + lane -----------------------------------------------
    if (warp < 4) {
        __syncwarp();
        bool have = mbar_wait(&s.accum, 0, p.status);
        asm volatile("tcgen05.fence::after_thread_sync;");
        const int64_t m = m0 + warp * 32 + lane;
        const bool partial = p.splits > 1;
        float *out = partial ? p.part + z * p.M * p.N : p.C + ob * p.sC;
        const int64_t ldo = partial ? p.N : p.ldc;
        for (int c0 = 0; c0 < TN; c0 += 16) {
            uint32_t r[16];
            uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (!have || m >= p.M) continue;
            float *row = out + m * ldo;
            for (int j = 0; j < 16; j++) {
                int64_t n = n0 + c0 + j;
                if (n >= p.N) break;
                float acc = __uint_as_float(r[j]);
                if (partial) {
                    row[n] = acc;
                } else {
                    float v = p.alpha * acc;
                    if (p.bias) v = v + (p.bias_row ? p.bias[m] : p.bias[n]);
                    if (p.beta != 0.0f) v = fmaf(p.beta, row[n], v);
                    row[n] = v;
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TN));
}

__global__ void k_tc_combine(TcParams p, int64_t nout) {
    int64_t MN = p.M * p.N, total = nout * MN;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ob = t / MN, r = t - ob * MN, m = r / p.N, n = r - m * p.N;
        const float *src = p.part + ob * p.splits * MN + r;
        float s = 0.0f;
        for (int k = 0; k < p.splits; k++) s += src[k * MN];
        float *c = p.C + ob * p.sC + m * p.ldc + n;
        float v = p.alpha * s;
        if (p.bias) v = v + (p.bias_row ? p.bias[m] : p.bias[n]);
        if (p.beta != 0.0f) v = fmaf(p.beta, *c, v);
        *c = v;
    }
}

// ---- host side -------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static int tried = 0;
    if (!tried) {
        tried = 1;
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)f;
        cudaGetLastError();
    }
    return fn;
}

// operand view: `inner` elements contiguous (lda stride between outer rows), optional batch dim
bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
              int64_t bstride, int box_inner, int box_outer, bool mn_major) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)bstride * 4};
    cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    cuuint32_t rank = batch > 1 ? 3 : 2;
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int S, bool THREE>
size_t smem_bytes() {
    size_t base = (sizeof(Smem<S>) + 1023) & ~(size_t)1023;
    return 1024 + base + (THREE ? sizeof(SmemLo<S>) : 0);
}

constexpr int kStagesTf32 = 4, kStages3x = 3;

}  // namespace

// Returns 1 when the GEMM was launched on the tensor cores, 0 when its layout does not fit the TMA
// constraints (16-byte aligned bases and strides) and the caller should use the FFMA kernel.
extern "C" int nck_gemm_tc(nck_dev *d, const nck_gemm_args *a) {
    if (a->M <= 0 || a->N <= 0 || a->batch <= 0 || a->K <= 0) return 0;
    if (a->M > INT32_MAX || a->N > INT32_MAX || a->K > INT32_MAX || a->batch > INT32_MAX) return 0;
    int three = d->gemm_mode == NCK_GEMM_3XTF32;
    int a_mn = a->ta, b_mn = !a->tb;
    int a_bat = a->batch > 1 && a->sA != 0, b_bat = a->batch > 1 && a->sB != 0;
    if ((uintptr_t)a->A % 16 || (uintptr_t)a->B % 16 || a->lda % 4 || a->ldb % 4) return 0;
    if ((a_bat && a->sA % 4) || (b_bat && a->sB % 4)) return 0;
    CUtensorMap ma, mb;
    // A: K-major [M][K] (ta = 0) or MN-major [K][M]
    bool okA = !a_mn ? make_map(&ma, a->A, a->K, a->M, a->lda, a_bat ? a->batch : 1, a->sA, TK, TM, false)
                     : make_map(&ma, a->A, a->M, a->K, a->lda, a_bat ? a->batch : 1, a->sA, 32, TK, true);
    // B: op(B) is K x N; K-major when stored [N][K] (tb = 1), MN-major when stored [K][N]
    bool okB = !b_mn ? make_map(&mb, a->B, a->K, a->N, a->ldb, b_bat ? a->batch : 1, a->sB, TK, TN, false)
                     : make_map(&mb, a->B, a->N, a->K, a->ldb, b_bat ? a->batch : 1, a->sB, 32, TK, true);
    if (!okA || !okB) return 0;

    TcParams p;
    memset(&p, 0, sizeof p);
    p.M = a->M, p.N = a->N, p.K = a->K, p.alpha = a->alpha, p.beta = a->beta;
    p.C = a->C, p.ldc = a->ldc, p.sC = a->sC, p.bias = a->bias, p.bias_row = a->bias_per_row;
    p.batch = a->batch, p.reduce = a->reduce_batch && a->batch > 1;
    p.a_mn = a_mn, p.b_mn = b_mn, p.a_bat = a_bat, p.b_bat = b_bat, p.three = three, p.status = d->status;

    int64_t tiles = ((a->M + TM - 1) / TM) * ((a->N + TN - 1) / TN);
    int64_t nout = p.reduce ? 1 : a->batch;
    int64_t target = (int64_t)d->sm_count;
    int64_t maxpart = (int64_t)(d->scratch_bytes / sizeof(float)) / (a->M * a->N * nout);
    int64_t splits = 1;
    if (tiles * nout < target) {
        splits = (target + tiles * nout - 1) / (tiles * nout);
        int64_t cap = p.reduce ? a->batch : (a->K + 4 * TK - 1) / (4 * TK);
        if (splits > cap) splits = cap;
        if (splits > maxpart) splits = maxpart;
        if (splits < 1) splits = 1;
    }
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
    if (nout * splits > 65535) return 0;

    size_t smem = three ? smem_bytes<kStages3x, true>() : smem_bytes<kStagesTf32, false>();
    static int attr_set[2] = {0, 0};
    if (!attr_set[three]) {
        cudaError_t e = three ? cudaFuncSetAttribute(k_tcgemm<kStages3x, true>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                              : cudaFuncSetAttribute(k_tcgemm<kStagesTf32, false>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        attr_set[three] = 1;
    }
    double nA = a->sA ? (double)a->batch : 1.0, nB = a->sB ? (double)a->batch : 1.0;
    double nC = (double)nout * (a->beta != 0.0f ? 2.0 : 1.0);
    Scope sc(d, three ? "gemm_3xtf32_tc" : "gemm_tf32_tc", 2.0 * a->M * a->N * a->K * a->batch,
             4.0 * (nA * a->M * a->K + nB * a->K * a->N + nC * a->M * a->N));
    dim3 grid((unsigned)((a->N + TN - 1) / TN), (unsigned)((a->M + TM - 1) / TM), (unsigned)(nout * splits));
    if (three) k_tcgemm<kStages3x, true><<<grid, 192, smem, NCK_STREAM(d)>>>(ma, mb, p);
    else k_tcgemm<kStagesTf32, false><<<grid, 128, smem, NCK_STREAM(d)>>>(ma, mb, p);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
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
