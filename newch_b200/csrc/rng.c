/* The context's random stream: xoshiro256** seeded by splitmix64, exactly as newch
 * (engine/src/core/ctx.c:270-276 seeding, :414-435 generator and float conversions), so initial
 * weights and dropout masks equal newch's for the same seed and call order.
 *
 * Dropout draws happen on the device. The xoshiro256** state transition is linear over GF(2), so
 * advancing the 256-bit state by k draws is a multiplication by the 256x256 bit matrix T^k. The
 * host keeps T^(2^i) for i < 64 (built once per process by repeated squaring) to skip its own
 * state past the draws a kernel consumed, and uploads T^(2^i) for i in [6, 42) to the device, where
 * the dropout kernel jumps each thread to the start of its 64-draw run.
 *
 * Bit matrices are stored by column: column j (4 x 64 bits) is the image of the state with only bit
 * j set. Bit j of the state is bit (j % 64) of word j / 64.
 */
#include "nc_internal.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static inline void step(uint64_t *s) {
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
}

uint64_t nc__rng_next(nc_ctx *ctx) {
    uint64_t *s = ctx->rng;
    uint64_t r = rotl64(s[1] * 5, 7) * 9;
    step(s);
    return r;
}

float nc__rand_uniform01(nc_ctx *ctx) { return (float)(nc__rng_next(ctx) >> 40) * (1.0f / 16777216.0f); }

float nc__rand_normal(nc_ctx *ctx) {
    float u1 = nc__rand_uniform01(ctx), u2 = nc__rand_uniform01(ctx);
    if (u1 < 1e-7f) u1 = 1e-7f;
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

/* ---- GF(2) jump matrices ------------------------------------------------------------------------ */

typedef uint64_t bitmat[256][4];

static bitmat *g_pow;      /* g_pow[i] = T^(2^i), i < 64 */
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void matvec(const bitmat m, const uint64_t *v, uint64_t *out) {
    uint64_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    for (int w = 0; w < 4; w++) {
        uint64_t bits = v[w];
        while (bits) {
            int b = __builtin_ctzll(bits);
            bits &= bits - 1;
            const uint64_t *c = m[w * 64 + b];
            a0 ^= c[0];
            a1 ^= c[1];
            a2 ^= c[2];
            a3 ^= c[3];
        }
    }
    out[0] = a0, out[1] = a1, out[2] = a2, out[3] = a3;
}

static void build_powers(void) {
    bitmat *p = (bitmat *)malloc(sizeof(bitmat) * 64);
    if (!p) return;
    for (int j = 0; j < 256; j++) {
        uint64_t s[4] = {0, 0, 0, 0};
        s[j / 64] = 1ull << (j % 64);
        step(s);
        memcpy(p[0][j], s, sizeof s);
    }
    for (int i = 1; i < 64; i++)
        for (int j = 0; j < 256; j++) matvec(p[i - 1], p[i - 1][j], p[i][j]); /* (T^k)^2 column j */
    g_pow = p;
}

static int powers_ready(void) {
    pthread_once(&g_once, build_powers);
    return g_pow != NULL;
}

void nc__rng_skip(nc_ctx *ctx, uint64_t n) {
    if (!n) return;
    if (n < 64 || !powers_ready()) {
        for (uint64_t i = 0; i < n; i++) step(ctx->rng);
        return;
    }
    uint64_t v[4];
    memcpy(v, ctx->rng, sizeof v);
    for (int i = 0; i < 64; i++) {
        if (!((n >> i) & 1)) continue;
        uint64_t o[4];
        matvec(g_pow[i], v, o);
        memcpy(v, o, sizeof v);
    }
    memcpy(ctx->rng, v, sizeof v);
}

/* device copies of T^(2^i), i in [6, 42): 36 matrices, 8 KiB each */
#define NC_RNG_POW_LO 6
#define NC_RNG_POW_N 36

int nc__rng_device_init(nc_ctx *ctx) {
    if (!powers_ready()) {
        nc__error(ctx, NC_ERR_OOM, "out of host memory (rng tables)");
        return 0;
    }
    if (nck_rng_tables_upload(nc__k(ctx), &g_pow[NC_RNG_POW_LO][0][0], sizeof(bitmat) * NC_RNG_POW_N) != 0) {
        nc__error(ctx, NC_ERR_STATE, "could not upload the dropout jump tables");
        return 0;
    }
    return 1;
}
