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

// gx[n, j] += sum over b with idx[b] == n of g[b, j], rows b added in ascending order (newch adds
// them in that order; no atomics). Block (n, column chunk): the block scans the indices 256 at a
// time, compacts the positions that point at row n (a warp ballot, then a prefix over the warps keeps
// them in order) and every thread adds those rows' values in its column. The indices are read once
// per destination row from L2; the gradient rows once in all.
__global__ void __launch_bounds__(256) k_index_select_bwd(const float *__restrict__ g, const int32_t *__restrict__ idx,
                                                          float *__restrict__ gx, int64_t B, int64_t N, int64_t row) {
    __shared__ int32_t hits[256];
    __shared__ int warp_base[9];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t j = blockIdx.y * (int64_t)blockDim.x + threadIdx.x;
    for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
        float acc = j < row ? gx[n * row + j] : 0.0f;
        for (int64_t b0 = 0; b0 < B; b0 += blockDim.x) {
            const int64_t b = b0 + threadIdx.x;
            const bool hit = b < B && __ldg(idx + b) == (int32_t)n;
            const unsigned mask = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) warp_base[warp + 1] = __popc(mask);
            __syncthreads();
            if (threadIdx.x == 0) {
                warp_base[0] = 0;
                for (int w = 1; w <= (int)(blockDim.x >> 5); w++) warp_base[w] += warp_base[w - 1];
            }
            __syncthreads();
            if (hit) hits[warp_base[warp] + __popc(mask & ((1u << lane) - 1u))] = (int32_t)(b - b0);
            __syncthreads();
            const int count = warp_base[blockDim.x >> 5];
            if (j < row)
                for (int k = 0; k < count; k++) acc += __ldg(g + (b0 + hits[k]) * row + j);
            __syncthreads(); // hits and warp_base are rewritten by the next chunk
        }
        if (j < row) gx[n * row + j] = acc;
    }
}

extern "C" void nck_index_select_bwd(nck_dev *d, const float *g, const int32_t *idx, float *gx, int64_t B, int64_t N,
                                     int64_t row) {
    if (B <= 0 || N * row <= 0) return;
    Scope sc(d, "index_select_bwd", 0.0, 4.0 * (B * row + 2 * N * row) + 4.0 * B);
    const int64_t chunks = (row + 255) / 256;
    int64_t rows = N < 65535 ? N : 65535;
    dim3 grid((unsigned)rows, (unsigned)chunks);
    k_index_select_bwd<<<grid, 256, 0, NCK_STREAM(d)>>>(g, idx, gx, B, N, row);
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
