/* Context: device binding, device step arena, persistent device memory, host step arena for
 * headers, error model, xoshiro256** RNG, host<->device copies.
 *
 * Arena policy follows newch (engine/src/core/ctx.c:128-339): bump allocation, a best-fit list of
 * blocks released during backward (at most 1/4 slack), O(1) reset at step end. On the device the
 * chunks are large (>= 64 MiB, doubling) stream-ordered pool allocations, so a steady-state step
 * never calls the allocator; block headers live in host memory because the device memory itself
 * cannot hold them.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

static size_t align_up(size_t v, size_t a) { return (v + (a - 1)) & ~(a - 1); }

/* ---- errors ------------------------------------------------------------------------------------ */

void nc__error(nc_ctx *ctx, nc_status code, const char *fmt, ...) {
    if (!ctx || ctx->status != NC_OK) return;
    ctx->status = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->err, sizeof ctx->err, fmt, ap);
    va_end(ap);
}

int nc__cuda_ok(nc_ctx *ctx, int err, const char *what) {
    if (err == cudaSuccess) return 1;
    nc__error(ctx, err == cudaErrorMemoryAllocation ? NC_ERR_OOM : NC_ERR_STATE, "%s: CUDA error %d (%s)", what, err,
              cudaGetErrorString((cudaError_t)err));
    return 0;
}

int nc__sync(nc_ctx *ctx) {
    if (!ctx->device_ok) return 0;
    nc__dp_join(ctx); /* gradient reduces on the communication stream finish first */
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)ctx->dev.stream);
    if (!nc__cuda_ok(ctx, e, "stream synchronize")) return 0;
    int code = *(volatile int *)ctx->dev.status_host;
    if (code != NCK_OK) {
        *(volatile int *)ctx->dev.status_host = NCK_OK;
        if (code == NCK_ERR_LABEL) nc__error(ctx, NC_ERR_ARG, "a label is outside [0, C) (found on the device)");
        else if (code == NCK_ERR_INDEX) nc__error(ctx, NC_ERR_ARG, "an index is out of range (found on the device)");
        else if (code == NCK_ERR_PIPELINE)
            nc__error(ctx, NC_ERR_STATE, "a tensor-core pipeline wait timed out (kernel gave up, results invalid)");
        else nc__error(ctx, NC_ERR_STATE, "a kernel failed to launch");
        return 0;
    }
    return ctx->status == NC_OK;
}

int nc_ok(const nc_ctx *ctx) { return ctx->status == NC_OK; }
nc_status nc_status_code(const nc_ctx *ctx) { return ctx->status; }
const char *nc_error(const nc_ctx *ctx) { return ctx->status == NC_OK ? "" : ctx->err; }
void nc_clear_error(nc_ctx *ctx) {
    ctx->status = NC_OK;
    ctx->err[0] = '\0';
}

/* ---- host step arena (headers, nodes, records) ------------------------------------------------ */

void *nc__meta_alloc(nc_ctx *ctx, size_t bytes, int persistent) {
    if (persistent) {
        void *p = calloc(1, bytes ? bytes : 1);
        if (!p) nc__error(ctx, NC_ERR_OOM, "out of host memory (%zu bytes)", bytes);
        return p;
    }
    size_t need = align_up(bytes ? bytes : 1, NC_HOST_ALIGN);
    nc_hchunk *c = ctx->hcur;
    while (c && c->cap - c->used < need) c = c->next;
    if (!c) {
        size_t cap = need > NC_HOST_CHUNK ? need : NC_HOST_CHUNK;
        c = (nc_hchunk *)malloc(sizeof(nc_hchunk) + NC_HOST_ALIGN + cap);
        if (!c) {
            nc__error(ctx, NC_ERR_OOM, "out of host memory (%zu bytes)", bytes);
            return NULL;
        }
        c->next = NULL;
        c->cap = cap;
        c->used = 0;
        c->base = (unsigned char *)align_up((size_t)(uintptr_t)(c + 1), NC_HOST_ALIGN);
        if (!ctx->hchunks) ctx->hchunks = c;
        else {
            nc_hchunk *t = ctx->hchunks;
            while (t->next) t = t->next;
            t->next = c;
        }
    }
    void *p = c->base + c->used;
    c->used += need;
    ctx->hcur = c;
    memset(p, 0, bytes);
    return p;
}

void nc__meta_free(nc_ctx *ctx, void *p, int persistent) {
    (void)ctx;
    if (persistent) free(p);
}

/* ---- device step arena ------------------------------------------------------------------------ */

static void log_temp(nc_ctx *ctx, void *p, size_t need) {
    if (!ctx->bwd_logging || ctx->grad_alloc || ctx->bwd_tmp_n >= 64) return;
    ctx->bwd_tmp[ctx->bwd_tmp_n] = p;
    ctx->bwd_tmp_size[ctx->bwd_tmp_n++] = need;
}

static void *reuse_block(nc_ctx *ctx, size_t need) {
    int best = -1;
    for (int i = 0; i < ctx->n_dfree; i++) {
        size_t sz = ctx->dfree[i].size;
        if (sz >= need && sz <= need + need / 4 && (best < 0 || sz < ctx->dfree[best].size)) {
            best = i;
            if (sz == need) break;
        }
    }
    if (best < 0) return NULL;
    nc_dfree b = ctx->dfree[best];
    ctx->dfree[best] = ctx->dfree[--ctx->n_dfree];
    ctx->arena_in_use += b.size;
    if (ctx->arena_in_use > ctx->arena_peak) ctx->arena_peak = ctx->arena_in_use;
    return b.p;
}

void *nc__arena_alloc(nc_ctx *ctx, size_t bytes) {
    size_t need = align_up(bytes ? bytes : 1, NC_DEV_ALIGN);
    if (!ctx->device_ok) {
        nc__error(ctx, NC_ERR_STATE, "no CUDA device: the B200 engine cannot allocate tensors");
        return NULL;
    }
    void *r = ctx->n_dfree ? reuse_block(ctx, need) : NULL;
    if (r) {
        log_temp(ctx, r, need);
        return r;
    }
    int i = ctx->cur_dchunk;
    while (i < ctx->n_dchunks && ctx->dchunks[i].cap - ctx->dchunks[i].used < need) i++;
    if (i == ctx->n_dchunks) {
        size_t cap = ctx->dchunk_min;
        if (ctx->n_dchunks) {
            size_t last = ctx->dchunks[ctx->n_dchunks - 1].cap;
            if (last * 2 > cap) cap = last * 2;
            if (cap > ((size_t)8 << 30)) cap = (size_t)8 << 30;
        }
        if (cap < need) cap = align_up(need, (size_t)2 << 20);
        void *p = NULL;
        cudaError_t e = cudaMallocAsync(&p, cap, (cudaStream_t)ctx->dev.stream);
        if (e != cudaSuccess) {
            cudaGetLastError();
            nc__error(ctx, NC_ERR_OOM, "out of device memory (arena, %zu bytes)", bytes);
            return NULL;
        }
        if (ctx->n_dchunks == ctx->cap_dchunks) {
            int nc = ctx->cap_dchunks ? ctx->cap_dchunks * 2 : 8;
            nc_dchunk *a = (nc_dchunk *)realloc(ctx->dchunks, sizeof(nc_dchunk) * (size_t)nc);
            if (!a) {
                nc__error(ctx, NC_ERR_OOM, "out of host memory");
                return NULL;
            }
            ctx->dchunks = a;
            ctx->cap_dchunks = nc;
        }
        ctx->dchunks[ctx->n_dchunks].base = (char *)p;
        ctx->dchunks[ctx->n_dchunks].cap = cap;
        ctx->dchunks[ctx->n_dchunks].used = 0;
        ctx->n_dchunks++;
        ctx->arena_reserved += cap;
    }
    nc_dchunk *c = &ctx->dchunks[i];
    void *p = c->base + c->used;
    c->used += need;
    ctx->cur_dchunk = i;
    ctx->arena_in_use += need;
    if (ctx->arena_in_use > ctx->arena_peak) ctx->arena_peak = ctx->arena_in_use;
    log_temp(ctx, p, need);
    return p;
}

void nc__arena_free(nc_ctx *ctx, void *p, size_t bytes) {
    if (!p) return;
    size_t size = align_up(bytes ? bytes : 1, NC_DEV_ALIGN);
    if (ctx->n_dfree == ctx->cap_dfree) {
        int nc = ctx->cap_dfree ? ctx->cap_dfree * 2 : 64;
        nc_dfree *a = (nc_dfree *)realloc(ctx->dfree, sizeof(nc_dfree) * (size_t)nc);
        if (!a) return; /* the block stays unused until step end */
        ctx->dfree = a;
        ctx->cap_dfree = nc;
    }
    ctx->dfree[ctx->n_dfree].p = (char *)p;
    ctx->dfree[ctx->n_dfree].size = size;
    ctx->n_dfree++;
    ctx->arena_in_use -= size;
}

/* Persistent device blocks are tracked in an open-addressing set (device memory cannot carry a
 * header), so nc_free_ctx can return every one of them. */
static size_t pmem_slot(const nc_ctx *ctx, const void *p) {
    uint64_t h = (uint64_t)(uintptr_t)p * 0x9E3779B97F4A7C15ull;
    return (size_t)(h >> 17) & (ctx->pmem_cap - 1);
}

static int pmem_insert(nc_ctx *ctx, void *p) {
    if ((ctx->pmem_n + 1) * 2 > ctx->pmem_cap) {
        size_t ncap = ctx->pmem_cap ? ctx->pmem_cap * 2 : 1024;
        void **old = ctx->pmem;
        size_t ocap = ctx->pmem_cap;
        ctx->pmem = (void **)calloc(ncap, sizeof(void *));
        if (!ctx->pmem) {
            ctx->pmem = old;
            return 0;
        }
        ctx->pmem_cap = ncap;
        for (size_t i = 0; i < ocap; i++) {
            if (!old[i] || old[i] == (void *)1) continue;
            size_t j = pmem_slot(ctx, old[i]);
            while (ctx->pmem[j]) j = (j + 1) & (ncap - 1);
            ctx->pmem[j] = old[i];
        }
        free(old);
    }
    size_t j = pmem_slot(ctx, p);
    while (ctx->pmem[j] && ctx->pmem[j] != (void *)1) j = (j + 1) & (ctx->pmem_cap - 1);
    ctx->pmem[j] = p;
    ctx->pmem_n++;
    return 1;
}

static void pmem_remove(nc_ctx *ctx, void *p) {
    if (!ctx->pmem_cap) return;
    size_t j = pmem_slot(ctx, p);
    while (ctx->pmem[j]) {
        if (ctx->pmem[j] == p) {
            ctx->pmem[j] = (void *)1; /* tombstone */
            ctx->pmem_n--;
            return;
        }
        j = (j + 1) & (ctx->pmem_cap - 1);
    }
}

void *nc__persistent_alloc(nc_ctx *ctx, size_t bytes) {
    if (!ctx->device_ok) {
        nc__error(ctx, NC_ERR_STATE, "no CUDA device: the B200 engine cannot allocate tensors");
        return NULL;
    }
    size_t need = align_up(bytes ? bytes : 1, NC_DEV_ALIGN);
    void *p = NULL;
    cudaError_t e = cudaMallocAsync(&p, need, (cudaStream_t)ctx->dev.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        nc__error(ctx, NC_ERR_OOM, "out of device memory (persistent, %zu bytes)", bytes);
        return NULL;
    }
    if (!pmem_insert(ctx, p)) {
        cudaFreeAsync(p, (cudaStream_t)ctx->dev.stream);
        nc__error(ctx, NC_ERR_OOM, "out of host memory");
        return NULL;
    }
    ctx->persistent_bytes += bytes;
    return p;
}

void nc__persistent_free(nc_ctx *ctx, void *p, size_t bytes) {
    if (!p) return;
    pmem_remove(ctx, p);
    cudaFreeAsync(p, (cudaStream_t)ctx->dev.stream);
    ctx->persistent_bytes -= bytes;
}

void *nc__alloc(nc_ctx *ctx, size_t bytes, int persistent) {
    return persistent ? nc__persistent_alloc(ctx, bytes) : nc__arena_alloc(ctx, bytes);
}

int nc__is_persistent_mode(const nc_ctx *ctx) { return ctx->persistent_depth > 0; }

/* ---- host <-> device copies ------------------------------------------------------------------- */

#define NC_STAGE_BYTES ((size_t)16 << 20)
#define NC_STAGE_SLOTS 32

void nc__upload(nc_ctx *ctx, void *dst, const void *src, size_t bytes) {
    nc__upload_on(ctx, ctx->dev.stream, dst, src, bytes);
}

void nc__upload_on(nc_ctx *ctx, void *stream, void *dst, const void *src, size_t bytes) {
    if (!bytes || !ctx->device_ok) return;
    cudaStream_t s = (cudaStream_t)stream;
    size_t slot_bytes = ctx->stage_cap / NC_STAGE_SLOTS;
    if (ctx->stage && bytes <= slot_bytes) {
        /* small uploads go through a pinned ring so the caller's buffer is free on return and
         * the copy stays asynchronous */
        int slot = ctx->stage_slot;
        ctx->stage_slot = (slot + 1) % NC_STAGE_SLOTS;
        cudaEventSynchronize((cudaEvent_t)ctx->stage_events[slot]);
        unsigned char *buf = ctx->stage + (size_t)slot * slot_bytes;
        memcpy(buf, src, bytes);
        nc__cuda_ok(ctx, cudaMemcpyAsync(dst, buf, bytes, cudaMemcpyHostToDevice, s), "upload");
        cudaEventRecord((cudaEvent_t)ctx->stage_events[slot], s);
        return;
    }
    struct cudaPointerAttributes at;
    int pinned = cudaPointerGetAttributes(&at, src) == cudaSuccess && at.type == cudaMemoryTypeHost;
    cudaGetLastError();
    nc__cuda_ok(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "upload");
    /* pageable sources are staged by the driver before the call returns; a pinned source is read
     * by the DMA engine later, so wait for it (the caller may reuse the buffer right away) */
    if (pinned) cudaStreamSynchronize(s);
}

void nc__download(nc_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!bytes || !ctx->device_ok) return;
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    if (!nc__cuda_ok(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "download")) return;
    nc__sync(ctx);
}

/* ---- lifecycle -------------------------------------------------------------------------------- */

static uint64_t splitmix64(uint64_t *x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* FP32 contraction mode. Default 3xTF32 on tcgen05 (hi*hi + hi*lo + lo*hi with fp32 accumulation:
 * fp32-class results at tensor-core speed); NC_GEMM=tf32 trades accuracy (rel ~1e-3) for a third of
 * the MMAs; NC_GEMM=ffma (and force_reference) selects the CUDA-core kernel whose per-element
 * summation order is fixed. */
static int gemm_mode_from_env(int force_reference) {
    if (force_reference) return NCK_GEMM_FFMA;
    const char *m = getenv("NC_GEMM");
    if (!m || !*m) return NCK_GEMM_3XTF32;
    if (!strcmp(m, "tf32")) return NCK_GEMM_TF32;
    if (!strcmp(m, "ffma")) return NCK_GEMM_FFMA;
    return NCK_GEMM_3XTF32;
}

int nc__dp_env_init(nc_ctx *ctx); /* dp.c */

nc_ctx *nc_init(const nc_config *cfg) {
    nc_ctx *ctx = (nc_ctx *)calloc(1, sizeof(nc_ctx));
    if (!ctx) return NULL;
    nc_config c;
    memset(&c, 0, sizeof c);
    if (cfg) c = *cfg;
    ctx->grad_enabled = 1;
    ctx->dp_world = 1;
    nc_manual_seed(ctx, c.seed);
    nc__detect_cpu(&ctx->cpu);
    ctx->n_threads = c.threads > 0 ? c.threads : ctx->cpu.n_cores;
    if (ctx->n_threads < 1) ctx->n_threads = 1;
    if (ctx->n_threads > 64) ctx->n_threads = 64;
    ctx->force_reference = c.force_reference;
    ctx->dchunk_min = c.arena_chunk_bytes > NC_MIN_DEV_CHUNK ? c.arena_chunk_bytes : NC_MIN_DEV_CHUNK;

    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) {
        cudaGetLastError();
        snprintf(ctx->device_name, sizeof ctx->device_name, "none");
        nc__error(ctx, NC_ERR_STATE, "no CUDA device visible: the B200 engine has no CPU fallback");
        return ctx;
    }
    const char *dv = getenv("NC_DEVICE");
    int dev = dv && *dv ? atoi(dv) : 0;
    if (dev < 0 || dev >= ndev) dev = 0;
    if (!nc__cuda_ok(ctx, cudaSetDevice(dev), "cudaSetDevice")) return ctx;
    struct cudaDeviceProp prop;
    if (!nc__cuda_ok(ctx, cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties")) return ctx;
    snprintf(ctx->device_name, sizeof ctx->device_name, "%.120s", prop.name);
    ctx->dev.device = dev;
    ctx->dev.sm_count = prop.multiProcessorCount;
    ctx->dev.gemm_mode = gemm_mode_from_env(c.force_reference);
    {
        const char *cv = getenv("NC_CONV");
        ctx->dev.conv_implicit = cv && !strcmp(cv, "implicit");
        ctx->dev.conv_tap = !cv || !strcmp(cv, "tap");
        const char *gs = getenv("NC_GEMM_SMALL");
        ctx->dev.gemm_small = !gs || strcmp(gs, "0") != 0;
        const char *qg = getenv("NC_QGEMM");
        ctx->dev.qgemm_tc = !qg || strcmp(qg, "dp4a") != 0;
        /* BatchNorm channel reductions fed by bulk copies: by default the statistics pass over planes of
         * at least 4 KiB (measured faster there); NC_BN_BULK=0 never, =8 / =16 every eligible pass in
         * 8 / 16 KiB stages */
        const char *bb = getenv("NC_BN_BULK");
        ctx->dev.bn_bulk_stage = !bb ? -16384 : !strcmp(bb, "0") ? 0 : !strcmp(bb, "8") ? 8192 : 16384;
        /* exp / sigmoid / tanh / erf: newch's AVX2-tier polynomials unless the reference tier's C
         * library forms are asked for (force_reference, as newch selects its reference tier) */
        const char *fz = getenv("NC_FUSE");
        ctx->fuse = !fz || strcmp(fz, "0") != 0;
        const char *mm = getenv("NC_MATH");
        ctx->dev.math_mode = (c.force_reference || (mm && !strcmp(mm, "libm"))) ? NCK_MATH_LIBM : NCK_MATH_POLY;
    }
    cudaStream_t s;
    if (!nc__cuda_ok(ctx, cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return ctx;
    ctx->dev.stream = s;
    /* keep freed pool memory cached: persistent frees and arena trims are re-used, not returned */
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t thr = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
    cudaGetLastError();
    void *st = NULL;
    if (!nc__cuda_ok(ctx, cudaHostAlloc(&st, 64, cudaHostAllocMapped), "status word")) return ctx;
    memset(st, 0, 64);
    void *st_dev = NULL;
    if (!nc__cuda_ok(ctx, cudaHostGetDevicePointer(&st_dev, st, 0), "status word")) return ctx;
    ctx->dev.status_host = (int *)st;
    ctx->dev.status = (int *)st_dev;
    ctx->dev.scratch_bytes = (size_t)64 << 20;
    if (!nc__cuda_ok(ctx, cudaMalloc(&ctx->dev.scratch, ctx->dev.scratch_bytes), "scratch")) return ctx;
    if (!nc__cuda_ok(ctx, cudaMalloc((void **)&ctx->dev.counters, 256), "counters")) return ctx;
    if (!nc__cuda_ok(ctx, cudaMemset(ctx->dev.counters, 0, 256), "counters")) return ctx;
    void *stage = NULL;
    if (cudaHostAlloc(&stage, NC_STAGE_BYTES, cudaHostAllocDefault) == cudaSuccess) {
        ctx->stage = (unsigned char *)stage;
        ctx->stage_cap = NC_STAGE_BYTES;
        for (int i = 0; i < NC_STAGE_SLOTS; i++) {
            cudaEvent_t ev;
            cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
            ctx->stage_events[i] = ev;
        }
    }
    cudaGetLastError();
    ctx->device_ok = 1;
    if (!nc__rng_device_init(ctx)) return ctx;
    nc__dp_env_init(ctx);
    return ctx;
}

void nc_manual_seed(nc_ctx *ctx, uint64_t seed) {
    uint64_t s = seed ? seed : 0x6E63u;
    for (int i = 0; i < 4; i++) ctx->rng[i] = splitmix64(&s);
    ctx->rng_count = ctx->rng_step_start = 0;
}

void nc__dp_free(nc_ctx *ctx); /* dp.c */

void nc_free_ctx(nc_ctx *ctx) {
    if (!ctx) return;
    if (ctx->device_ok) {
        cudaStream_t s = (cudaStream_t)ctx->dev.stream;
        cudaStreamSynchronize(s);
        nc__rng_side_free(ctx);
        nc__dp_free(ctx);
        for (int i = 0; i < ctx->n_dchunks; i++) cudaFreeAsync(ctx->dchunks[i].base, s);
        for (size_t i = 0; i < ctx->pmem_cap; i++)
            if (ctx->pmem[i] && ctx->pmem[i] != (void *)1) cudaFreeAsync(ctx->pmem[i], s);
        cudaStreamSynchronize(s);
        for (int i = 0; i < NC_STAGE_SLOTS; i++)
            if (ctx->stage_events[i]) cudaEventDestroy((cudaEvent_t)ctx->stage_events[i]);
        if (ctx->stage) cudaFreeHost(ctx->stage);
        if (ctx->dev.scratch) cudaFree(ctx->dev.scratch);
        if (ctx->dev.counters) cudaFree(ctx->dev.counters);
        if (ctx->dev.status_host) cudaFreeHost(ctx->dev.status_host);
        nck_timer_enable(&ctx->dev, 0);
        cudaStreamDestroy(s);
        cudaGetLastError();
    }
    /* persistent tensor headers are host mallocs owned by their callers' handles; the device
     * blocks were returned above */
    free(ctx->pmem);
    nc_hchunk *c = ctx->hchunks;
    while (c) {
        nc_hchunk *n = c->next;
        free(c);
        c = n;
    }
    free(ctx->dchunks);
    free(ctx->dfree);
    free(ctx);
}

void nc_step_end(nc_ctx *ctx) {
    nc__deferred_reset(ctx);
    nc__rng_side_step_end(ctx);
    if (ctx->bn_n) nc__dp_bn_flush(ctx, 0); /* statistics staged in a step no optimizer step closed */
    nc__dp_rng_step_end(ctx);
    for (int i = 0; i < ctx->n_dchunks; i++) ctx->dchunks[i].used = 0;
    ctx->cur_dchunk = 0;
    ctx->n_dfree = 0;
    ctx->arena_in_use = 0;
    for (nc_hchunk *c = ctx->hchunks; c; c = c->next) c->used = 0;
    ctx->hcur = ctx->hchunks;
    ctx->tape = NULL;
    ctx->bwd_tmp_n = 0;
}

void nc_arena_trim(nc_ctx *ctx) {
    if (!ctx->device_ok) return;
    cudaStream_t s = (cudaStream_t)ctx->dev.stream;
    int keep = 0;
    for (int i = 0; i < ctx->n_dchunks; i++) {
        if (ctx->dchunks[i].used == 0) {
            cudaFreeAsync(ctx->dchunks[i].base, s);
            ctx->arena_reserved -= ctx->dchunks[i].cap;
        } else {
            ctx->dchunks[keep++] = ctx->dchunks[i];
        }
    }
    ctx->n_dchunks = keep;
    ctx->cur_dchunk = 0;
    nc_hchunk **link = &ctx->hchunks;
    while (*link) {
        nc_hchunk *c = *link;
        if (c->used == 0) {
            *link = c->next;
            free(c);
        } else {
            link = &c->next;
        }
    }
    ctx->hcur = ctx->hchunks;
}

int nc_num_threads(const nc_ctx *ctx) { return ctx->n_threads; }
void nc_persistent_begin(nc_ctx *ctx) { ctx->persistent_depth++; }
void nc_persistent_end(nc_ctx *ctx) {
    if (ctx->persistent_depth > 0) ctx->persistent_depth--;
}

int nc_set_grad_enabled(nc_ctx *ctx, int enabled) {
    int prev = ctx->grad_enabled;
    ctx->grad_enabled = enabled ? 1 : 0;
    return prev;
}

nc_mem_stats nc_get_mem_stats(const nc_ctx *ctx) {
    nc_mem_stats s;
    s.persistent_bytes = ctx->persistent_bytes;
    s.arena_bytes_in_use = ctx->arena_in_use;
    s.arena_bytes_reserved = ctx->arena_reserved;
    s.arena_peak_bytes = ctx->arena_peak;
    return s;
}

void nc_reset_peak(nc_ctx *ctx) { ctx->arena_peak = ctx->arena_in_use; }

const nc_cpu_info *nc_cpu(const nc_ctx *ctx) { return &ctx->cpu; }
const char *nc_kernel_backend(const nc_ctx *ctx) {
    (void)ctx;
    return "b200";
}

/* ---- side API -------------------------------------------------------------------------------- */

int nc_ext_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

const char *nc_ext_device_name(const nc_ctx *ctx) { return ctx->device_name; }

int nc_ext_synchronize(nc_ctx *ctx) {
    nc__sync(ctx);
    return ctx->status;
}

int nc_ext_pipeline_wait_probe(nc_ctx *ctx) {
    if (!ctx->device_ok) return ctx->status;
    nck_pipeline_wait_probe(nc__k(ctx));
    nc__sync(ctx);
    return ctx->status;
}

int64_t nc_ext_launch_count(const nc_ctx *ctx) { return ctx->dev.launches; }

const char *nc_ext_gemm_mode(const nc_ctx *ctx) {
    switch (ctx->dev.gemm_mode) {
    case NCK_GEMM_TF32: return "tf32";
    case NCK_GEMM_3XTF32: return "3xtf32";
    default: return "ffma";
    }
}

void *nc_ext_stream(nc_ctx *ctx) { return ctx->dev.stream; }

int nc_ext_timing(nc_ctx *ctx, int on) {
    if (!ctx->device_ok) return NC_ERR_STATE;
    nck_timer_enable(&ctx->dev, on);
    return NC_OK;
}

int nc_ext_kernel_time(nc_ctx *ctx, const char *prefix, double *ms, int64_t *count) {
    if (!ctx->device_ok) return NC_ERR_STATE;
    nc__sync(ctx);
    return nck_timer_query(&ctx->dev, prefix ? prefix : "", ms, count);
}

int nc_ext_kernel_entry(nc_ctx *ctx, int i, const char **name, double *ms, int64_t *count, double *flops,
                        double *bytes) {
    if (!ctx->device_ok) return 0;
    nc__sync(ctx);
    return nck_timer_entry(&ctx->dev, i, name, ms, count, flops, bytes);
}

void nc_ext_timing_reset(nc_ctx *ctx) {
    if (!ctx->device_ok) return;
    nc__sync(ctx);
    nck_timer_reset(&ctx->dev);
}
