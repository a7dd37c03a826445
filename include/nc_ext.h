/*
 * nc_ext.h — side API of the B200 newch engine.
 *
 * These entry points have no counterpart in newch's engine/include/nc.h, whose ABI stays frozen.
 * They sit where newch plans its optional engine/src/ext/ module (newch CLAUDE.md:83-85): device
 * facts, data-parallel set-up (NCCL over NVLink/NVSwitch) and counters for benchmarks. A newch
 * user needs none of them: data parallelism can also be switched on purely through the
 * environment (NC_RANK, NC_WORLD_SIZE, NC_NCCL_ID_FILE), read by nc_init.
 */
#ifndef NC_EXT_H
#define NC_EXT_H

#include "nc.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Number of visible CUDA devices (0 when there is none or the driver is missing). */
NC_API int nc_ext_device_count(void);
/* Name of the context's device, e.g. "NVIDIA B200". */
NC_API const char *nc_ext_device_name(const nc_ctx *ctx);
/* Waits for all work enqueued by the context; returns its status code (kernel-found errors become
 * NC_ERR_ARG, CUDA failures NC_ERR_STATE). */
NC_API int nc_ext_synchronize(nc_ctx *ctx);
/* Kernels this context has enqueued since nc_init. */
NC_API int64_t nc_ext_launch_count(const nc_ctx *ctx);
/* "ffma", "tf32" or "3xtf32": how fp32 GEMMs run (NC_GEMM env; force_reference forces "ffma"). */
NC_API const char *nc_ext_gemm_mode(const nc_ctx *ctx);

/* Writes an NCCL unique id (bytes) into buf; returns its length or -1. Rank 0 calls it and sends
 * the bytes to the other ranks by any host channel. */
NC_API int nc_ext_nccl_unique_id(void *buf, int cap);
/* Joins the context to a data-parallel group of `world` ranks. After this, nc_optim_step averages
 * the gradients of all ranks (one all-reduce of the flat gradient buffer) before updating.
 * Returns NC_OK or an error status. */
NC_API int nc_ext_dp_init(nc_ctx *ctx, int rank, int world, const void *id, int id_len);
NC_API int nc_ext_dp_world(const nc_ctx *ctx);
/* Dropout streams of a data-parallel group that reproduce newch's gradient accumulation over the
 * ranks' batches (rank r's step draws what newch draws for the r-th micro-batch of an accumulated
 * step): every step of every rank takes at most `draws_per_step` random numbers, rank r starts r
 * strides into each step's span of world * draws_per_step draws, and nc_step_end moves it to its
 * place in the next span. Call after nc_ext_dp_init, at the point training starts. 0 turns the
 * interleaving off. Returns NC_OK or NC_ERR_ARG. */
NC_API int nc_ext_dp_rng_stride(nc_ctx *ctx, int64_t draws_per_step);
/* Random numbers taken from the context's stream since it was seeded. */
NC_API int64_t nc_ext_rng_position(const nc_ctx *ctx);

/* The cudaStream_t every kernel of this context runs on. */
NC_API void *nc_ext_stream(nc_ctx *ctx);
/* Per-kernel timing with CUDA events on the context's stream (costs a little per launch). */
NC_API int nc_ext_timing(nc_ctx *ctx, int on);
/* Sum of device milliseconds and the number of timed launches of kernels whose name starts with
 * `prefix` ("" = all) since timing was switched on. */
NC_API int nc_ext_kernel_time(nc_ctx *ctx, const char *prefix, double *ms, int64_t *count);
/* Timed kernel class i (0-based): its name, total device milliseconds, launches and the algorithmic
 * work of those launches (FLOPs, and bytes that must move: each logical input read once, each
 * output written once). Returns 0 when i is past the last class. */
NC_API int nc_ext_kernel_entry(nc_ctx *ctx, int i, const char **name, double *ms, int64_t *count, double *flops,
                               double *bytes);
/* Clears the accumulated timings (timing stays on). */
NC_API void nc_ext_timing_reset(nc_ctx *ctx);

/* Failure-reporting probe: launches one kernel whose tensor-core pipeline wait (an mbarrier that
 * never completes) gives up after its 2 s bound, as every tcgen05 kernel's waits do, then
 * synchronizes. Returns the context status: NC_ERR_STATE with "pipeline wait timed out" in
 * nc_error. The device stays usable: nc_clear_error and continue. */
NC_API int nc_ext_pipeline_wait_probe(nc_ctx *ctx);

/* Cross-entropy forward on caller-owned device buffers that allocates nothing. It has no
 * counterpart in newch; the arithmetic is the engine's nc_cross_entropy (newch
 * engine/src/ops/ops_nn.c:107-149): prob[rows, classes] = softmax(logits) and
 * *loss = -mean(log prob[r, labels[r]]), with the mean summed in double in a fixed order.
 *
 * For callers that must not have device memory allocated on their behalf while they run (a runtime
 * that owns and accounts for the whole device pool, a latency-critical loop, a process at its
 * memory limit): the only scratch is a static device array of NC_EXT_CE_NOALLOC_MAX_ROWS floats.
 * All pointers are device pointers; `stream` is a cudaStream_t (NULL = the legacy default stream).
 * The call is asynchronous. Returns NC_OK, NC_ERR_ARG (rows < 0, rows > NC_EXT_CE_NOALLOC_MAX_ROWS,
 * classes <= 0, or a NULL pointer; nothing is launched) or NC_ERR_STATE (CUDA set-up or launch
 * failure).
 * - The first call on a device (made with that device current) looks up the static array's address
 *   in the current CUDA context; a later call under another context (after cudaDeviceReset, say)
 *   looks it up again. Make such a first call before any stream capture begins.
 * - Launch failures are taken from the launches themselves: an error the caller left pending in the
 *   runtime's last-error slot is neither reported nor cleared.
 * - *status must start at zero; a label outside [0, classes) sets it to 2 (that row's label is
 *   read as class 0). The static array needs no initialisation.
 * - Calls on one device share the static array: calls that can run at the same time (on streams
 *   with no ordering between them) race on it. Calls ordered on one stream are safe. */
#define NC_EXT_CE_NOALLOC_MAX_ROWS 262144
NC_API int nc_ext_cross_entropy_fwd_noalloc(const float *logits, const int32_t *labels, int64_t rows,
                                            int64_t classes, float *prob, float *loss, int *status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NC_EXT_H */
