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
 *
 * Jumps by polynomial. T satisfies its characteristic polynomial P (degree 256, found once by
 * Berlekamp-Massey on 512 output bits of the generator), so T^d = q_d(T) with q_d = x^d mod P, a
 * 256-bit polynomial that does not depend on the state. The host keeps q_(64 k) for the runs of 64
 * draws the dropout kernel gives each thread (grown on demand, checked against the matrix jumps),
 * and a thread reaches its start state from the launch's state by Horner's rule: 256 generator
 * steps with a conditional XOR, independent of every other thread.
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
    ctx->rng_count++;
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
    ctx->rng_count += n;
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

/* ---- jump polynomials --------------------------------------------------------------------------- */

typedef uint64_t poly[4]; /* GF(2) polynomial of degree < 256: bit i = coefficient of x^i */

static poly g_charp;                       /* P(x) - x^256 */
static pthread_once_t g_charp_once = PTHREAD_ONCE_INIT;
static int g_charp_ok;

/* Berlekamp-Massey over GF(2) on the lowest output bit of the state's first word */
static void find_charpoly(void) {
    enum { NB = 512 };
    uint8_t a[NB];
    uint64_t s[4] = {0x9E3779B97F4A7C15ull, 0xBF58476D1CE4E5B9ull, 0x94D049BB133111EBull, 0x2545F4914F6CDD1Dull};
    for (int k = 0; k < NB; k++) {
        a[k] = (uint8_t)(s[0] & 1u);
        step(s);
    }
    uint8_t C[NB + 1] = {1}, B[NB + 1] = {1}, Tm[NB + 1];
    int L = 0, m = 1;
    for (int n = 0; n < NB; n++) {
        uint8_t dsc = a[n];
        for (int i = 1; i <= L; i++) dsc ^= (uint8_t)(C[i] & a[n - i]);
        if (!dsc) {
            m++;
        } else if (2 * L <= n) {
            memcpy(Tm, C, sizeof C);
            for (int i = 0; i + m <= NB; i++) C[i + m] ^= B[i];
            L = n + 1 - L;
            memcpy(B, Tm, sizeof B);
            m = 1;
        } else {
            for (int i = 0; i + m <= NB; i++) C[i + m] ^= B[i];
            m++;
        }
    }
    if (L != 256) return;
    /* a[k+256] = sum_j C[j] a[k+256-j]  =>  P(x) = x^256 + sum_{i<256} C[256-i] x^i */
    memset(g_charp, 0, sizeof g_charp);
    for (int i = 0; i < 256; i++)
        if (C[256 - i]) g_charp[i / 64] |= 1ull << (i % 64);
    g_charp_ok = 1;
}

/* a <- a * x mod P */
static inline void poly_mulx(uint64_t *a) {
    uint64_t top = a[3] >> 63;
    a[3] = (a[3] << 1) | (a[2] >> 63);
    a[2] = (a[2] << 1) | (a[1] >> 63);
    a[1] = (a[1] << 1) | (a[0] >> 63);
    a[0] <<= 1;
    if (top) a[0] ^= g_charp[0], a[1] ^= g_charp[1], a[2] ^= g_charp[2], a[3] ^= g_charp[3];
}

/* q(T) v by Horner: the same loop a device thread runs */
static void poly_apply(const uint64_t *q, const uint64_t *v, uint64_t *out) {
    uint64_t s[4], acc[4] = {0, 0, 0, 0};
    memcpy(s, v, sizeof s);
    for (int i = 0; i < 256; i++) {
        if ((q[i / 64] >> (i % 64)) & 1u) acc[0] ^= s[0], acc[1] ^= s[1], acc[2] ^= s[2], acc[3] ^= s[3];
        step(s);
    }
    memcpy(out, acc, sizeof acc);
}

static poly *g_runs;   /* g_runs[k] = x^(64 k) mod P */
static int64_t g_nruns, g_capruns;
static pthread_mutex_t g_runs_mu = PTHREAD_MUTEX_INITIALIZER;

/* x^(64 k) mod P for k < count (host copy, grown on demand); NULL when unavailable. The first call
 * checks a few polynomial jumps against the matrix jumps. */
const uint64_t *nc__rng_run_polys(int64_t count) {
    pthread_once(&g_charp_once, find_charpoly);
    if (!g_charp_ok || count <= 0 || !powers_ready()) return NULL;
    pthread_mutex_lock(&g_runs_mu);
    if (count > g_capruns || g_capruns < 8) {
        int64_t cap = g_capruns ? g_capruns : 1024;
        while (cap < count) cap *= 2;
        poly *r = (poly *)realloc(g_runs, (size_t)cap * sizeof(poly));
        if (!r) {
            pthread_mutex_unlock(&g_runs_mu);
            return NULL;
        }
        g_runs = r, g_capruns = cap;
    }
    int check = g_nruns == 0;
    if (count < 8) count = 8; /* the first call's check reads entries 1 and 5 */
    if (count > g_capruns) {
        pthread_mutex_unlock(&g_runs_mu);
        return NULL;
    }
    if (g_nruns == 0) {
        memset(g_runs[0], 0, sizeof(poly));
        g_runs[0][0] = 1;
        g_nruns = 1;
    }
    for (; g_nruns < count; g_nruns++) {
        memcpy(g_runs[g_nruns], g_runs[g_nruns - 1], sizeof(poly));
        for (int i = 0; i < 64; i++) poly_mulx(g_runs[g_nruns]);
    }
    if (check) {
        /* q_(64 k)(T) v must equal T^(64 k) v from the squared matrices */
        const uint64_t v[4] = {1, 0x1234567ull, 0xFEDCBA9876543210ull, 42};
        const int64_t ks[3] = {1, 5, count - 1};
        for (int t = 0; t < 3; t++) {
            uint64_t a[4], b[4], o[4];
            poly_apply(g_runs[ks[t]], v, a);
            memcpy(b, v, sizeof b);
            uint64_t d = (uint64_t)ks[t] * 64u;
            for (int i = 0; i < 64; i++) {
                if (!((d >> i) & 1)) continue;
                matvec(g_pow[i], b, o);
                memcpy(b, o, sizeof b);
            }
            if (memcmp(a, b, sizeof a)) {
                g_charp_ok = 0;
                pthread_mutex_unlock(&g_runs_mu);
                return NULL;
            }
        }
    }
    const uint64_t *out = &g_runs[0][0];
    pthread_mutex_unlock(&g_runs_mu);
    return out;
}

/* Device table of run polynomials covering n draws (runs of 64), uploaded once and grown on demand;
 * NULL when n is beyond the table's cap (2^27 draws) or the table is unavailable, and the dropout
 * kernel then jumps by matrices instead. */
/* The Horner window tables of the polynomial dropout kernel for the context's current state, on the
 * device: with the base states b_j = T^(64 j) s (j < 4), entry (j, w, v) is the XOR over the set
 * bits t of v of T^(4 w + t) b_j (w, v < 16), 32 bytes each, 32 KiB in all. T^i b_j is the state
 * 64 j + i steps past s, so 256 steps of a copy of the state give every term. Built here instead of
 * by a one-block kernel in front of every dropout launch; the block comes from the step arena and
 * reaches the device through the pinned staging ring. */
void nc__rng_build_tabs(const uint64_t s0[4], uint64_t (*tab)[4]) {
    uint64_t states[256][4]; /* 8 KiB */
    uint64_t st[4];
    memcpy(st, s0, sizeof st);
    for (int i = 0; i < 256; i++) {
        memcpy(states[i], st, sizeof st);
        step(st);
    }
    for (int e = 0; e < 4 * 16 * 16; e++) {
        const int j = e >> 8, w = (e >> 4) & 15, v = e & 15;
        uint64_t a[4] = {0, 0, 0, 0};
        for (int t = 0; t < 4; t++)
            if ((v >> t) & 1)
                for (int q = 0; q < 4; q++) a[q] ^= states[64 * j + 4 * w + t][q];
        memcpy(tab[e], a, sizeof a);
    }
}

const void *nc__rng_dropout_tabs(nc_ctx *ctx) {
    uint64_t tab[4 * 16 * 16][4]; /* 32 KiB, copied into the staging ring before the return */
    nc__rng_build_tabs(ctx->rng, tab);
    void *dev = nc__arena_alloc(ctx, sizeof tab);
    if (!dev) return NULL;
    nc__upload(ctx, dev, tab, sizeof tab);
    return dev;
}

const void *nc__rng_dropout_table(nc_ctx *ctx, int64_t n) {
    if (n <= 0 || n > ((int64_t)1 << 27)) return NULL;
    const char *jump = getenv("NC_DROPOUT_JUMP"); /* "matrix": always the matrix-jump kernel */
    if (jump && !strcmp(jump, "matrix")) return NULL;
    int64_t runs = (n + 63) / 64, want = 1024;
    while (want < runs) want *= 2;
    const uint64_t *host = nc__rng_run_polys(want);
    if (!host) return NULL;
    return nck_rng_polys(nc__k(ctx), host, want);
}
