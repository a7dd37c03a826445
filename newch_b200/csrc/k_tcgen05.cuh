// Device helpers shared by the tcgen05 kernels: mbarriers with bounded waits, shared-memory matrix
// and instruction descriptors for kind::tf32, MMA issue and commit, TMEM loads, the TF32 head/rest
// split. All functions are inline; each kernel family includes this header in its own file.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "k_common.cuh"

namespace tc {

using nck::report;

constexpr int TM = 128, TK = 32;          // tile rows (TMEM lanes); K per stage (32 fp32 = 128 B)
constexpr int kMaxBN = 128;               // widest tile
constexpr int kStageA = TM * TK;          // floats per lane-operand stage (16 KiB)
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kErrPipeline = 3;           // status code of a wait that gave up
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;        // dynamic shared memory per block on sm_100 (227 KiB)

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

// false when the bounded wait gave up (the error goes to the status word)
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

// K-offset descriptor of one stage buffer for the k-th 8-deep MMA step
__device__ __forceinline__ uint64_t stage_desc(uint32_t base, int mn, int k) {
    // K-major: 128 B rows of 32 K values, 8-row atoms 1024 B apart; step k moves 32 B along the row
    if (!mn) return sdesc(base + k * 32, 16, 1024, 2);
    // MN-major: 128 B rows of 32 M/N values, one row per K; 4-row atoms 512 B apart (SBO), 32-wide
    // blocks 4 KiB apart (LBO); step k moves 8 rows
    return sdesc(base + k * 1024, 4096, 512, 1);
}

// instruction descriptor: D f32, A/B tf32, dense, M = 128, N = bn
__device__ __forceinline__ uint32_t idesc_tf32(int a_mn, int b_mn, int bn) {
    uint32_t d = 0;
    d |= 1u << 4;               // D format F32
    d |= 2u << 7;               // A format TF32
    d |= 2u << 10;              // B format TF32
    d |= (uint32_t)a_mn << 15;  // A major
    d |= (uint32_t)b_mn << 16;  // B major
    d |= (uint32_t)(bn >> 3) << 17;
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

// TMA tile loads into shared memory (no multicast), completing on an mbarrier
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

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// The 3xTF32 remainder x - head, rounded to the nearest TF32 value (cvt.rna: ties away from zero).
// The tensor core truncates its operands, so an unrounded remainder would lose its own low 13 bits
// toward zero on every product, a bias that grows with the length of the reduction; a remainder that
// is already a TF32 value passes through exactly and its rounding error has no preferred sign.
__device__ __forceinline__ float tf32_rest(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x - tf32_hi(x)));
    return __uint_as_float(r);
}

__device__ __forceinline__ float4 tf32_rest4(float4 v) {
    return make_float4(tf32_rest(v.x), tf32_rest(v.y), tf32_rest(v.z), tf32_rest(v.w));
}

// 16 consecutive accumulator columns of this warp's 32 lanes (32x32b shape, one register per column)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMEM columns to allocate for two accumulators of bn columns (a power of two, at least 32, at most 512)
__host__ __device__ constexpr uint32_t tmem_cols(int bn) {
    return bn * 2 <= 32 ? 32 : bn * 2 <= 64 ? 64 : bn * 2 <= 128 ? 128 : bn * 2 <= 256 ? 256 : 512;
}

// tmem_ld16 without the wait: several loads in flight, then one tmem_wait_ld
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// waits for every tcgen05.ld of this thread; r (loaded before the wait) is tied to the wait so that
// no use of it is scheduled above it
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// ties registers loaded before an earlier tmem_wait_ld to a point after it (volatile asm keeps order)
__device__ __forceinline__ void tmem_regs_after_wait(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}

// instruction descriptor: D s32, A/B signed int8, K-major, M = 128, N = bn (kind::i8)
__device__ __forceinline__ uint32_t idesc_s8(int bn) {
    uint32_t d = 0;
    d |= 2u << 4;   // D format S32
    d |= 1u << 7;   // A signed 8-bit
    d |= 1u << 10;  // B signed 8-bit
    d |= (uint32_t)(bn >> 3) << 17;
    d |= (uint32_t)(TM >> 4) << 24;
    return d;
}

__device__ __forceinline__ void mma_s8(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// ---- host side: TMA tensor maps ------------------------------------------------------------------

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encoder() {
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

// operand view: `inner` elements contiguous (ld elements between outer rows), optional batch dim
inline bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
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
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// byte matrix (int8 / uint8) view: rows of `inner` bytes, `ld` bytes apart; 128-byte swizzle
inline bool make_map_u8(CUtensorMap *map, const void *base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                        int box_outer) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace tc
