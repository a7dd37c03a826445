/* Data parallelism: one process per GPU, one NCCL communicator per context, one all-reduce (mean)
 * of the optimizer's flat gradient buffer per update. newch has no distributed code; the contract
 * here is that N ranks stepping on N micro-batches give the update newch computes with
 * gradient_accumulation_steps = N over the same micro-batches (engine/src/optim/optim.c:161-167).
 *
 * Set-up: nc_ext_dp_init with an id from nc_ext_nccl_unique_id, or the environment read by nc_init:
 * NC_RANK, NC_WORLD_SIZE and NC_NCCL_ID_FILE (rank 0 writes the id there, the others wait for it,
 * bounded by NC_DP_TIMEOUT seconds, default 120; the file carries the launch's token,
 * NC_NCCL_ID_TOKEN or torchrun's TORCHELASTIC_RUN_ID, and ranks ignore a file with another token). Communicator errors are polled with a deadline
 * and end in ncclCommAbort, so a dead peer surfaces as NC_ERR_STATE instead of a hang.
 */
#define _POSIX_C_SOURCE 200809L
#include "nc_internal.h"

#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <time.h>
#include <unistd.h>

/* NCCL is opened on first use, not linked: a process that never joins a data-parallel group never
 * loads it, and a process that also hosts another NCCL user (a framework that bundles its own
 * libnccl.so.2) shares whichever copy that user loaded first instead of pinning an older one. */
static struct {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
    int ok;
} nccl_fn;
static pthread_once_t nccl_once = PTHREAD_ONCE_INIT;

static void nccl_open(void) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define NC_NCCL_SYM(field, name) *(void **)&nccl_fn.field = dlsym(h, name)
    NC_NCCL_SYM(GetUniqueId, "ncclGetUniqueId");
    NC_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    NC_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    NC_NCCL_SYM(CommAbort, "ncclCommAbort");
    NC_NCCL_SYM(CommDestroy, "ncclCommDestroy");
    NC_NCCL_SYM(AllReduce, "ncclAllReduce");
    NC_NCCL_SYM(AllGather, "ncclAllGather");
    NC_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef NC_NCCL_SYM
    nccl_fn.ok = nccl_fn.GetUniqueId && nccl_fn.CommInitRankConfig && nccl_fn.CommGetAsyncError &&
                 nccl_fn.CommAbort && nccl_fn.CommDestroy && nccl_fn.AllReduce && nccl_fn.AllGather &&
                 nccl_fn.GetErrorString;
}

static int nccl_loaded(void) {
    pthread_once(&nccl_once, nccl_open);
    return nccl_fn.ok;
}

#define ncclGetUniqueId(...) (nccl_loaded() ? nccl_fn.GetUniqueId(__VA_ARGS__) : ncclSystemError)
#define ncclCommInitRankConfig(...) (nccl_loaded() ? nccl_fn.CommInitRankConfig(__VA_ARGS__) : ncclSystemError)
#define ncclCommGetAsyncError(...) (nccl_loaded() ? nccl_fn.CommGetAsyncError(__VA_ARGS__) : ncclSystemError)
#define ncclCommAbort(...) (nccl_loaded() ? nccl_fn.CommAbort(__VA_ARGS__) : ncclSystemError)
#define ncclCommDestroy(...) (nccl_loaded() ? nccl_fn.CommDestroy(__VA_ARGS__) : ncclSystemError)
#define ncclAllReduce(...) (nccl_loaded() ? nccl_fn.AllReduce(__VA_ARGS__) : ncclSystemError)
#define ncclAllGather(...) (nccl_loaded() ? nccl_fn.AllGather(__VA_ARGS__) : ncclSystemError)
#define ncclGetErrorString(r) (nccl_loaded() ? nccl_fn.GetErrorString(r) : "libnccl.so.2 could not be loaded")

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static double timeout_s(void) {
    const char *v = getenv("NC_DP_TIMEOUT");
    double t = v && *v ? atof(v) : 120.0;
    return t > 0 ? t : 120.0;
}

int nc_ext_nccl_unique_id(void *buf, int cap) {
    ncclUniqueId id;
    if (cap < (int)sizeof id || ncclGetUniqueId(&id) != ncclSuccess) return -1;
    memcpy(buf, &id, sizeof id);
    return (int)sizeof id;
}

/* Waits for an NCCL call issued in non-blocking mode; aborts the communicator past the deadline. A
 * collective's enqueue usually finishes within microseconds, and the step's critical path waits for it,
 * so the state is polled back to back for the first ~2 ms and with short sleeps after that (a sleep
 * per poll added ~0.2 ms to every gradient bucket). */
static int comm_wait(nc_ctx *ctx, ncclComm_t comm, const char *what) {
    const double start = now_s(), deadline = start + timeout_s();
    int spin = 1;
    for (unsigned i = 0;; i++) {
        ncclResult_t st = ncclInProgress;
        if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return 1;
        if (spin && (i & 255) == 255 && now_s() - start > 2e-3) spin = 0;
        if (st != ncclInProgress || (!spin && now_s() > deadline)) {
            ncclCommAbort(comm);
            ctx->nccl_comm = NULL;
            ctx->dp_world = 1;
            nc__error(ctx, NC_ERR_STATE, "%s: NCCL %s", what,
                      st == ncclInProgress ? "timed out (a peer did not join)" : ncclGetErrorString(st));
            return 0;
        }
        if (!spin) usleep(50);
    }
}

int nc_ext_dp_init(nc_ctx *ctx, int rank, int world, const void *id, int id_len) {
    if (!ctx->device_ok) return NC_ERR_STATE;
    if (world < 1 || rank < 0 || rank >= world || id_len != (int)sizeof(ncclUniqueId)) {
        nc__error(ctx, NC_ERR_ARG, "dp_init: rank %d / world %d / id of %d bytes", rank, world, id_len);
        return NC_ERR_ARG;
    }
    if (world == 1) return NC_OK;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = NULL;
    ncclResult_t r = ncclCommInitRankConfig(&comm, world, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        nc__error(ctx, NC_ERR_STATE, "dp_init: ncclCommInitRank failed: %s", ncclGetErrorString(r));
        return NC_ERR_STATE;
    }
    ctx->nccl_comm = comm;
    ctx->dp_world = world;
    ctx->dp_rank = rank;
    if (!comm_wait(ctx, comm, "dp_init")) return ctx->status;
    /* gradient buckets are all-reduced on their own stream, overlapping the rest of the backward */
    cudaStream_t cs = NULL;
    cudaEvent_t e1 = NULL, e2 = NULL;
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if (!nc__cuda_ok(ctx, cudaStreamCreateWithPriority(&cs, cudaStreamNonBlocking, hi), "comm stream") ||
        !nc__cuda_ok(ctx, cudaEventCreateWithFlags(&e1, cudaEventDisableTiming), "comm event") ||
        !nc__cuda_ok(ctx, cudaEventCreateWithFlags(&e2, cudaEventDisableTiming), "comm event"))
        return ctx->status;
    ctx->comm_stream = cs;
    ctx->ev_main = e1;
    ctx->ev_comm = e2;
    return NC_OK;
}

int nc_ext_dp_world(const nc_ctx *ctx) { return ctx->dp_world; }

/* The id file written by rank 0: a header naming the run, then the NCCL id. Ranks > 0 accept only a
 * file of their own run, so a file left by an earlier run at the same path is never joined. */
typedef struct {
    char magic[8]; /* "NCDPID1" */
    char token[56];
    ncclUniqueId id;
} dp_id_file;

/* the launch's token: NC_NCCL_ID_TOKEN, else torchrun's per-launch run id, else none */
static const char *run_token(void) {
    const char *t = getenv("NC_NCCL_ID_TOKEN");
    if (!t || !*t) t = getenv("TORCHELASTIC_RUN_ID");
    return t && *t ? t : "";
}

int nc__dp_env_init(nc_ctx *ctx) {
    const char *ws = getenv("NC_WORLD_SIZE"), *rk = getenv("NC_RANK"), *file = getenv("NC_NCCL_ID_FILE");
    if (!ws || !rk || !file) return 1;
    int world = atoi(ws), rank = atoi(rk);
    if (world <= 1) return 1;
    dp_id_file rec;
    memset(&rec, 0, sizeof rec);
    memcpy(rec.magic, "NCDPID1", 8);
    snprintf(rec.token, sizeof rec.token, "%s", run_token());
    if (rank == 0) {
        if (nc_ext_nccl_unique_id(&rec.id, sizeof rec.id) < 0) {
            nc__error(ctx, NC_ERR_STATE, "dp: ncclGetUniqueId failed");
            return 0;
        }
        char tmp[4096];
        snprintf(tmp, sizeof tmp, "%s.tmp", file);
        FILE *f = fopen(tmp, "wb");
        if (!f || fwrite(&rec, sizeof rec, 1, f) != 1) {
            if (f) fclose(f);
            nc__error(ctx, NC_ERR_STATE, "dp: cannot write %s", tmp);
            return 0;
        }
        fclose(f);
        rename(tmp, file); /* appears atomically for the other ranks */
    } else {
        double deadline = now_s() + timeout_s();
        for (;;) {
            FILE *f = fopen(file, "rb");
            if (f) {
                dp_id_file got;
                size_t n = fread(&got, 1, sizeof got, f);
                fclose(f);
                if (n == sizeof got && !memcmp(got.magic, rec.magic, 8) &&
                    !strncmp(got.token, rec.token, sizeof rec.token)) {
                    rec.id = got.id;
                    break;
                }
            }
            if (now_s() > deadline) {
                nc__error(ctx, NC_ERR_STATE, "dp: rank %d gave up waiting for %s (run token \"%s\")", rank, file,
                          rec.token);
                return 0;
            }
            usleep(10000);
        }
    }
    return nc_ext_dp_init(ctx, rank, world, &rec.id, sizeof rec.id) == NC_OK;
}

int nc__dp_allreduce_mean(nc_ctx *ctx, float *buf, int64_t n) {
    if (ctx->dp_world <= 1 || !n) return 1;
    ncclComm_t comm = (ncclComm_t)ctx->nccl_comm;
    if (!comm) {
        nc__error(ctx, NC_ERR_STATE, "dp: no communicator");
        return 0;
    }
    ncclResult_t r = ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclAvg, comm, (cudaStream_t)ctx->dev.stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        nc__error(ctx, NC_ERR_STATE, "dp: ncclAllReduce failed: %s", ncclGetErrorString(r));
        return 0;
    }
    if (r == ncclInProgress) return comm_wait(ctx, comm, "all-reduce");
    return 1;
}

static int enqueue_on_comm(nc_ctx *ctx, const void *src, void *dst, int64_t n, ncclDataType_t type,
                           ncclRedOp_t op, const char *what) {
    if (ctx->dp_world <= 1 || n <= 0) return 1;
    ncclComm_t comm = (ncclComm_t)ctx->nccl_comm;
    if (!comm || !ctx->comm_stream) {
        nc__error(ctx, NC_ERR_STATE, "dp: no communicator");
        return 0;
    }
    cudaStream_t cs = (cudaStream_t)ctx->comm_stream;
    cudaEventRecord((cudaEvent_t)ctx->ev_main, (cudaStream_t)ctx->dev.stream);
    cudaStreamWaitEvent(cs, (cudaEvent_t)ctx->ev_main, 0);
    ncclResult_t r = ncclAllReduce(src, dst, (size_t)n, type, op, comm, cs);
    if (r != ncclSuccess && r != ncclInProgress) {
        nc__error(ctx, NC_ERR_STATE, "dp: %s failed: %s", what, ncclGetErrorString(r));
        return 0;
    }
    if (r == ncclInProgress && !comm_wait(ctx, comm, what)) return 0;
    ctx->comm_pending = 1;
    return 1;
}

int nc__dp_reduce_async(nc_ctx *ctx, const float *src, float *dst, int64_t n) {
    return enqueue_on_comm(ctx, src, dst, n, ncclFloat32, ncclAvg, "gradient all-reduce");
}

int nc__dp_max_bytes_async(nc_ctx *ctx, unsigned char *buf, int64_t n) {
    return enqueue_on_comm(ctx, buf, buf, n, ncclUint8, ncclMax, "presence all-reduce");
}

void nc__dp_join(nc_ctx *ctx) {
    if (!ctx->comm_pending || !ctx->comm_stream) return;
    cudaEventRecord((cudaEvent_t)ctx->ev_comm, (cudaStream_t)ctx->comm_stream);
    cudaStreamWaitEvent((cudaStream_t)ctx->dev.stream, (cudaEvent_t)ctx->ev_comm, 0);
    ctx->comm_pending = 0;
}

/* ---- BatchNorm running statistics under data parallelism ------------------------------------------ */

typedef struct nc_bn_pending {
    float *rm, *rv;
    int64_t C, off;
    float mom;
} nc_bn_pending;

#define NC_BN_STAGE_FLOATS ((int64_t)1 << 20)

float *nc__dp_bn_stage(nc_ctx *ctx, float *running_mean, float *running_var, int64_t C, float momentum) {
    if (2 * C > NC_BN_STAGE_FLOATS) {
        nc__error(ctx, NC_ERR_ARG, "batch_norm: %lld channels exceed the data-parallel staging area",
                  (long long)C);
        return NULL;
    }
    if (!ctx->bn_stage) {
        ctx->bn_stage = (float *)nc__persistent_alloc(ctx, sizeof(float) * (size_t)NC_BN_STAGE_FLOATS);
        ctx->bn_gather = (float *)nc__persistent_alloc(ctx, sizeof(float) * (size_t)NC_BN_STAGE_FLOATS *
                                                                (size_t)ctx->dp_world);
        if (!ctx->bn_stage || !ctx->bn_gather) return NULL;
        ctx->bn_stage_cap = NC_BN_STAGE_FLOATS;
    }
    /* a step that stages more than the area holds applies what it has first (every rank does the same) */
    if (ctx->bn_stage_used + 2 * C > ctx->bn_stage_cap && !nc__dp_bn_flush(ctx, 0)) return NULL;
    if (ctx->bn_n == ctx->bn_cap) {
        int cap = ctx->bn_cap ? 2 * ctx->bn_cap : 32;
        nc_bn_pending *p = (nc_bn_pending *)realloc(ctx->bn_pending, sizeof(nc_bn_pending) * (size_t)cap);
        if (!p) {
            nc__error(ctx, NC_ERR_OOM, "batch_norm: out of host memory");
            return NULL;
        }
        ctx->bn_pending = p;
        ctx->bn_cap = cap;
    }
    nc_bn_pending *e = &ctx->bn_pending[ctx->bn_n++];
    e->rm = running_mean, e->rv = running_var, e->C = C, e->mom = momentum, e->off = ctx->bn_stage_used;
    ctx->bn_stage_used += (2 * C + 3) & ~(int64_t)3;
    return ctx->bn_stage + e->off;
}

/* Gathers every rank's staged statistics and applies the updates (one NCCL all-gather and one
 * kernel per flush), on the communication stream (joined by the caller) or on the main stream. */
int nc__dp_bn_flush(nc_ctx *ctx, int on_comm_stream) {
    if (!ctx->bn_n) return 1;
    if (ctx->dp_world <= 1 || !ctx->nccl_comm) {
        nc__error(ctx, NC_ERR_STATE, "batch_norm: statistics staged without a data-parallel group");
        return 0;
    }
    /* table: groups of forwards sharing a running-statistics pair, each group in recording order */
    int n = ctx->bn_n;
    size_t bytes = sizeof(nck_bn_group) * (size_t)n + sizeof(nck_bn_staged) * (size_t)n;
    if (ctx->bn_table_cap < n) {
        if (ctx->bn_table_dev)
            nc__persistent_free(ctx, ctx->bn_table_dev,
                                (sizeof(nck_bn_group) + sizeof(nck_bn_staged)) * (size_t)ctx->bn_table_cap);
        ctx->bn_table_dev = nc__persistent_alloc(ctx, bytes);
        if (!ctx->bn_table_dev) return 0;
        ctx->bn_table_cap = n;
    }
    unsigned char *host = (unsigned char *)malloc(bytes);
    int *used = (int *)calloc((size_t)n, sizeof(int));
    if (!host || !used) {
        free(host);
        free(used);
        nc__error(ctx, NC_ERR_OOM, "batch_norm: out of host memory");
        return 0;
    }
    nck_bn_group *groups = (nck_bn_group *)host;
    nck_bn_staged *staged = (nck_bn_staged *)(host + sizeof(nck_bn_group) * (size_t)n);
    int ng = 0, ns = 0;
    for (int i = 0; i < n; i++) {
        if (used[i]) continue;
        nck_bn_group *g = &groups[ng++];
        g->rm = ctx->bn_pending[i].rm, g->rv = ctx->bn_pending[i].rv, g->C = ctx->bn_pending[i].C;
        g->e0 = ns;
        for (int j = i; j < n; j++) {
            if (used[j] || ctx->bn_pending[j].rm != g->rm) continue;
            used[j] = 1;
            staged[ns].off = ctx->bn_pending[j].off;
            staged[ns].mom = ctx->bn_pending[j].mom;
            staged[ns].pad = 0;
            ns++;
        }
        g->e1 = ns;
    }
    unsigned char *dev = (unsigned char *)ctx->bn_table_dev;
    nc__upload(ctx, dev, groups, sizeof(nck_bn_group) * (size_t)ng);
    nc__upload(ctx, dev + sizeof(nck_bn_group) * (size_t)n, staged, sizeof(nck_bn_staged) * (size_t)ns);
    free(host);
    free(used);

    cudaStream_t st = (cudaStream_t)ctx->dev.stream;
    if (on_comm_stream) {
        st = (cudaStream_t)ctx->comm_stream;
        cudaEventRecord((cudaEvent_t)ctx->ev_main, (cudaStream_t)ctx->dev.stream);
        cudaStreamWaitEvent(st, (cudaEvent_t)ctx->ev_main, 0);
        ctx->comm_pending = 1;
    }
    ncclComm_t comm = (ncclComm_t)ctx->nccl_comm;
    ncclResult_t r = ncclAllGather(ctx->bn_stage, ctx->bn_gather, (size_t)ctx->bn_stage_used, ncclFloat32, comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
        nc__error(ctx, NC_ERR_STATE, "dp: BatchNorm statistics all-gather failed: %s", ncclGetErrorString(r));
        return 0;
    }
    if (r == ncclInProgress && !comm_wait(ctx, comm, "BatchNorm statistics all-gather")) return 0;
    nck_dev d = ctx->dev;
    d.stream = st;
    nck_bn_running_apply(&d, (const nck_bn_group *)dev, ng, (const nck_bn_staged *)(dev + sizeof(nck_bn_group) * (size_t)n),
                         ctx->bn_gather, ctx->bn_stage_used, ctx->dp_world);
    ctx->dev.launches = d.launches;
    ctx->bn_n = 0;
    ctx->bn_stage_used = 0;
    return 1;
}

/* ---- dropout streams under data parallelism -------------------------------------------------------- */

int nc_ext_dp_rng_stride(nc_ctx *ctx, int64_t draws_per_step) {
    if (!ctx) return NC_ERR_ARG;
    if (draws_per_step < 0) {
        nc__error(ctx, NC_ERR_ARG, "dp_rng_stride: draws per step must be >= 0, got %lld", (long long)draws_per_step);
        return NC_ERR_ARG;
    }
    ctx->dp_rng_stride = ctx->dp_world > 1 ? draws_per_step : 0;
    if (ctx->dp_rng_stride) nc__rng_skip(ctx, (uint64_t)ctx->dp_rank * (uint64_t)draws_per_step);
    ctx->rng_step_start = ctx->rng_count;
    return NC_OK;
}

int64_t nc_ext_rng_position(const nc_ctx *ctx) { return ctx ? (int64_t)ctx->rng_count : 0; }

void nc__dp_rng_step_end(nc_ctx *ctx) {
    if (ctx->dp_world <= 1 || ctx->dp_rng_stride <= 0) return;
    const uint64_t D = (uint64_t)ctx->dp_rng_stride, used = ctx->rng_count - ctx->rng_step_start;
    if (used > D) {
        nc__error(ctx, NC_ERR_STATE, "dp: a step drew %llu random numbers, more than the stride of %llu",
                  (unsigned long long)used, (unsigned long long)D);
        return;
    }
    /* to the start of this rank's micro-batch in the next step: the other ranks' draws come between */
    nc__rng_skip(ctx, (uint64_t)ctx->dp_world * D - used);
    ctx->rng_step_start = ctx->rng_count;
}

void nc__dp_free(nc_ctx *ctx) {
    if (ctx->comm_stream) cudaStreamSynchronize((cudaStream_t)ctx->comm_stream);
    if (ctx->nccl_comm) {
        ncclCommDestroy((ncclComm_t)ctx->nccl_comm);
        ctx->nccl_comm = NULL;
    }
    free(ctx->bn_pending);
    ctx->bn_pending = NULL;
    if (ctx->ev_main) cudaEventDestroy((cudaEvent_t)ctx->ev_main);
    if (ctx->ev_comm) cudaEventDestroy((cudaEvent_t)ctx->ev_comm);
    if (ctx->comm_stream) cudaStreamDestroy((cudaStream_t)ctx->comm_stream);
    ctx->ev_main = ctx->ev_comm = ctx->comm_stream = NULL;
}
