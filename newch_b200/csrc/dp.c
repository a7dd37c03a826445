/* Data parallelism: one process per GPU, one NCCL communicator per context, one all-reduce (mean)
 * of the optimizer's flat gradient buffer per update. newch has no distributed code; the contract
 * here is that N ranks stepping on N micro-batches give the update newch computes with
 * gradient_accumulation_steps = N over the same micro-batches (engine/src/optim/optim.c:161-167).
 *
 * Set-up: nc_ext_dp_init with an id from nc_ext_nccl_unique_id, or the environment read by nc_init:
 * NC_RANK, NC_WORLD_SIZE and NC_NCCL_ID_FILE (rank 0 writes the id there, the others wait for it,
 * bounded by NC_DP_TIMEOUT seconds, default 120). Communicator errors are polled with a deadline
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
    NC_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef NC_NCCL_SYM
    nccl_fn.ok = nccl_fn.GetUniqueId && nccl_fn.CommInitRankConfig && nccl_fn.CommGetAsyncError &&
                 nccl_fn.CommAbort && nccl_fn.CommDestroy && nccl_fn.AllReduce && nccl_fn.GetErrorString;
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

/* Waits for an NCCL call issued in non-blocking mode; aborts the communicator past the deadline. */
static int comm_wait(nc_ctx *ctx, ncclComm_t comm, const char *what) {
    double deadline = now_s() + timeout_s();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return 1;
        if (st != ncclInProgress || now_s() > deadline) {
            ncclCommAbort(comm);
            ctx->nccl_comm = NULL;
            ctx->dp_world = 1;
            nc__error(ctx, NC_ERR_STATE, "%s: NCCL %s", what,
                      st == ncclInProgress ? "timed out (a peer did not join)" : ncclGetErrorString(st));
            return 0;
        }
        usleep(200);
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
    return NC_OK;
}

int nc_ext_dp_world(const nc_ctx *ctx) { return ctx->dp_world; }

int nc__dp_env_init(nc_ctx *ctx) {
    const char *ws = getenv("NC_WORLD_SIZE"), *rk = getenv("NC_RANK"), *file = getenv("NC_NCCL_ID_FILE");
    if (!ws || !rk || !file) return 1;
    int world = atoi(ws), rank = atoi(rk);
    if (world <= 1) return 1;
    ncclUniqueId id;
    if (rank == 0) {
        if (nc_ext_nccl_unique_id(&id, sizeof id) < 0) {
            nc__error(ctx, NC_ERR_STATE, "dp: ncclGetUniqueId failed");
            return 0;
        }
        char tmp[4096];
        snprintf(tmp, sizeof tmp, "%s.tmp", file);
        FILE *f = fopen(tmp, "wb");
        if (!f || fwrite(&id, sizeof id, 1, f) != 1) {
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
                size_t got = fread(&id, 1, sizeof id, f);
                fclose(f);
                if (got == sizeof id) break;
            }
            if (now_s() > deadline) {
                nc__error(ctx, NC_ERR_STATE, "dp: rank %d gave up waiting for %s", rank, file);
                return 0;
            }
            usleep(10000);
        }
    }
    return nc_ext_dp_init(ctx, rank, world, &id, sizeof id) == NC_OK;
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

void nc__dp_free(nc_ctx *ctx) {
    if (ctx->nccl_comm) {
        ncclCommDestroy((ncclComm_t)ctx->nccl_comm);
        ctx->nccl_comm = NULL;
    }
}
