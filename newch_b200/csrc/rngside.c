/* Dropout keep masks drawn on a side stream.
 *
 * A dropout's mask depends only on the generator's state at the call (known on the host), not on any
 * tensor. Drawing it is integer work (state jumps and steps) of the same order as the whole dropout,
 * so it is launched on a second stream the moment the call is made: the GPU is usually still running
 * earlier kernels of the step on the main stream, and the draw overlaps them. The main stream waits
 * for the mask right before the kernel that applies it (y = x * mask / (1 - p), or the fused
 * attention kernel), so values are those of the single-stream path bit for bit.
 *
 * Memory: the masks and their window tables come from a side pool (a bump allocator over one device
 * block, reset at nc_step_end), never from the step arena, whose blocks the main stream may still be
 * reading when the side stream would write them. The first draw of a step waits for an event that
 * nc_step_end records on the main stream, so a step's masks never overwrite the previous step's while
 * its backward still reads them. With per-kernel timing on (the benchmark's kernel table), for masks
 * under NC_SIDE_MIN_DRAWS (unless NC_RNG_SIDE=1), with NC_RNG_SIDE=0, or when the pool is full, masks
 * are drawn on the main stream instead.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

#define NC_SIDE_POOL_BYTES ((size_t)64 << 20)
#define NC_SIDE_TABS_BYTES ((size_t)4 * 16 * 16 * 32)

/* Masks below this many draws are drawn on the main stream by the fused draw-and-apply kernel: one
 * launch and no events, where the host's cost of the side path (tables, events, two launches) exceeded
 * the overlap it buys (cfg2's 64k-draw mask: 2.7% slower with it; cfg4's 2-8M-draw masks: 3.3% faster). */
#define NC_SIDE_MIN_DRAWS ((int64_t)1 << 20)

static int side_ready(nc_ctx *ctx, int64_t n) {
    if (ctx->side_off || !ctx->device_ok) return 0;
    if (!ctx->side_stream) {
        const char *e = getenv("NC_RNG_SIDE"); /* 0: never, 1: every mask, unset: masks of >= 1M draws */
        if (e && !strcmp(e, "0")) {
            ctx->side_off = 1;
            return 0;
        }
        ctx->side_all = e && !strcmp(e, "1");
    }
    if (n < NC_SIDE_MIN_DRAWS && !ctx->side_all) return 0;
    if (ctx->side_stream) return 1;
    cudaStream_t s = NULL;
    cudaEvent_t a = NULL, b = NULL;
    void *pool = NULL;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&a, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&b, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&pool, NC_SIDE_POOL_BYTES) != cudaSuccess) {
        cudaGetLastError();
        if (pool) cudaFree(pool);
        if (b) cudaEventDestroy(b);
        if (a) cudaEventDestroy(a);
        if (s) cudaStreamDestroy(s);
        ctx->side_off = 1;
        return 0;
    }
    ctx->side_stream = s, ctx->ev_side = a, ctx->ev_step = b;
    ctx->side_pool = (unsigned char *)pool, ctx->side_cap = NC_SIDE_POOL_BYTES, ctx->side_used = 0;
    ctx->side_fresh = 1;
    return 1;
}

static void *side_alloc(nc_ctx *ctx, size_t bytes) {
    const size_t at = (ctx->side_used + 255) & ~(size_t)255;
    if (at + bytes > ctx->side_cap) return NULL;
    ctx->side_used = at + bytes;
    return ctx->side_pool + at;
}

int nc__rng_side_mask(nc_ctx *ctx, int64_t n, float p, uint32_t **bits) {
    if (n <= 0 || ctx->dev.timer || !side_ready(ctx, n)) return 0;
    const void *polys = nc__rng_dropout_table(ctx, n);
    if (!polys) return 0; /* beyond the polynomial tables: the main-stream kernel jumps by matrices */
    const size_t words = (size_t)(n + 31) / 32 + 1;
    const size_t mark = ctx->side_used;
    void *tabs = side_alloc(ctx, NC_SIDE_TABS_BYTES);
    uint32_t *b = (uint32_t *)side_alloc(ctx, words * sizeof(uint32_t));
    if (!tabs || !b) {
        ctx->side_used = mark;
        return 0;
    }
    cudaStream_t side = (cudaStream_t)ctx->side_stream, main = (cudaStream_t)ctx->dev.stream;
    if (ctx->side_fresh) { /* the previous step's readers of the pool are done */
        cudaStreamWaitEvent(side, (cudaEvent_t)ctx->ev_step, 0);
        ctx->side_fresh = 0;
    }
    uint64_t tab[4 * 16 * 16][4];
    nc__rng_build_tabs(ctx->rng, tab);
    nc__upload_on(ctx, side, tabs, tab, sizeof tab);
    nck_dev d = *nc__k(ctx);
    d.stream = side;
    nck_dropout_fwd(&d, ctx->rng, NULL, NULL, b, n, p, polys, tabs);
    ctx->dev.launches += d.launches - nc__k(ctx)->launches;
    if (!nc__cuda_ok(ctx, cudaEventRecord((cudaEvent_t)ctx->ev_side, side), "side stream") ||
        !nc__cuda_ok(ctx, cudaStreamWaitEvent(main, (cudaEvent_t)ctx->ev_side, 0), "side stream"))
        return 0;
    *bits = b;
    return 1;
}

void nc__rng_side_step_end(nc_ctx *ctx) {
    if (!ctx->side_stream) return;
    cudaEventRecord((cudaEvent_t)ctx->ev_step, (cudaStream_t)ctx->dev.stream);
    ctx->side_used = 0;
    ctx->side_fresh = 1;
}

void nc__rng_side_free(nc_ctx *ctx) {
    if (!ctx->side_stream) return;
    cudaStreamSynchronize((cudaStream_t)ctx->side_stream);
    cudaFree(ctx->side_pool);
    cudaEventDestroy((cudaEvent_t)ctx->ev_side);
    cudaEventDestroy((cudaEvent_t)ctx->ev_step);
    cudaStreamDestroy((cudaStream_t)ctx->side_stream);
    ctx->side_stream = NULL;
    ctx->side_pool = NULL;
}
