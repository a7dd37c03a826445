// Row gathers and their gradients: index_select along axis 0 (batch gathering, embedding lookup),
// and the row-interleaving copies of cat.
#include "k_common.cuh"

using namespace nck;

// y[b, :] = x[idx[b], :]; rows moved with 16-byte words when the row size allows
__global__ void k_index_select(const char *__restrict__ x, const int32_t *__restrict__ idx, char *__restrict__ y,
                               int64_t B, int64_t N, int64_t row_bytes, int *status) {
    int vec = (row_bytes & 15) == 0 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    int64_t units = vec ? row_bytes / 16 : row_bytes;
    int64_t total = B * units;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = t / units, u = t - b * units;
        int64_t r = idx[b];
        if (r < 0 || r >= N) {
            report(status, NCK_ERR_INDEX);
            continue;
        }
        if (vec) ((int4 *)(y + b * row_bytes))[u] = ((const int4 *)(x + r * row_bytes))[u];
        else y[b * row_bytes + u] = x[r * row_bytes + u];
    }
}

extern "C" void nck_index_select(nck_dev *d, const void *x, const int32_t *idx, void *y, int64_t B, int64_t N,
                                 int64_t row_bytes) {
    if (B <= 0 || row_bytes <= 0) return;
    Scope sc(d, "index_select", 0.0, 2.0 * B * row_bytes + 4.0 * B);
    int64_t units = (row_bytes & 15) == 0 ? row_bytes / 16 : row_bytes;
    k_index_select<<<grid_for(d, B * units), kThreads, 0, NCK_STREAM(d)>>>((const char *)x, idx, (char *)y, B, N,
                                                                           row_bytes, d->status);
    NCK_LAUNCHED(d, 1);
}

// gx[n, j] += sum over b with idx[b] == n of g[b, j], rows b visited in order (no atomics):
// one thread per (n, j); for a small table (an embedding of 96 rows) every thread scans the indices
__global__ void k_index_select_bwd(const float *__restrict__ g, const int32_t *__restrict__ idx, float *__restrict__ gx,
                                   int64_t B, int64_t N, int64_t row) {
    extern __shared__ int32_t sidx[];
    int64_t total = N * row;
    for (int64_t t0 = blockIdx.x * (int64_t)blockDim.x; t0 < total; t0 += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = t0 + threadIdx.x;
        int64_t n = t / row, j = t - n * row;
        float acc = t < total ? gx[t] : 0.0f;
        for (int64_t b0 = 0; b0 < B; b0 += 2048) {
            int64_t nb = B - b0 < 2048 ? B - b0 : 2048;
            __syncthreads();
            for (int64_t k = threadIdx.x; k < nb; k += blockDim.x) sidx[k] = idx[b0 + k];
            __syncthreads();
            if (t < total)
                for (int64_t k = 0; k < nb; k++)
                    if (sidx[k] == n) acc += g[(b0 + k) * row + j];
        }
        if (t < total) gx[t] = acc;
    }
}

extern "C" void nck_index_select_bwd(nck_dev *d, const float *g, const int32_t *idx, float *gx, int64_t B, int64_t N,
                                     int64_t row) {
    if (B <= 0 || N * row <= 0) return;
    Scope sc(d, "index_select_bwd");
    k_index_select_bwd<<<grid_for(d, N * row), kThreads, 2048 * sizeof(int32_t), NCK_STREAM(d)>>>(g, idx, gx, B, N,
                                                                                                   row);
    NCK_LAUNCHED(d, 1);
}

// cat: each input's rows land at their column offset of the output rows (one 2-D copy)
extern "C" void nck_cat_part(nck_dev *d, const void *x, void *y, int64_t outer, int64_t row_bytes,
                             int64_t out_row_bytes, int64_t off_bytes) {
    if (outer * row_bytes <= 0) return;
    Scope sc(d, "cat");
    cudaMemcpy2DAsync((char *)y + off_bytes, (size_t)out_row_bytes, x, (size_t)row_bytes, (size_t)row_bytes,
                      (size_t)outer, cudaMemcpyDeviceToDevice, NCK_STREAM(d));
}

__global__ void k_cat_part_bwd(const float *__restrict__ g, float *__restrict__ gx, int64_t outer, int64_t row,
                               int64_t out_row, int64_t off) {
    int64_t total = outer * row;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / row, j = t - o * row;
        gx[t] = fmaf(1.0f, g[o * out_row + off + j], gx[t]);
    }
}

extern "C" void nck_cat_part_bwd(nck_dev *d, const float *g, float *gx, int64_t outer, int64_t row, int64_t out_row,
                                 int64_t off) {
    if (outer * row <= 0) return;
    Scope sc(d, "cat_bwd");
    k_cat_part_bwd<<<grid_for(d, outer * row), kThreads, 0, NCK_STREAM(d)>>>(g, gx, outer, row, out_row, off);
    NCK_LAUNCHED(d, 1);
}
