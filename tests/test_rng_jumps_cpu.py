"""The engine's host-side jump arithmetic for the dropout stream (newch_b200/csrc/rng.c), on CPU.

rng.c finds the characteristic polynomial P of the xoshiro256** transition T by Berlekamp-Massey and
keeps q_k = x^(64 k) mod P; the dropout kernel reaches the start of run k as q_k(T) s0, with q_k split
into four 64-bit words r_j evaluated on the base states T^(64 j) s0 (Horner's rule over 4-bit
windows on the device). This test compiles rng.c with stubs for its device calls and checks, against
plain sequential stepping of the generator (the reference's own stream, engine/src/core/ctx.c:414-435):
P has degree 256, q_k(T) v = T^(64 k) v for runs near the start and far into a 2^20-draw tensor, and
the four-word split with base states gives the same state, as do the host-built 4-bit window tables
the kernel reads (nc__rng_dropout_tabs)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent

HARNESS = r"""
#include "rng.c"
#include <stdio.h>
int nck_rng_tables_upload(nck_dev *d, const uint64_t *t, size_t b) { return 0; }
const void *nck_rng_polys(nck_dev *d, const uint64_t *h, int64_t c) { return 0; }
void nc__error(nc_ctx *ctx, nc_status st, const char *fmt, ...) {}
static uint64_t g_arena[1024][4], g_dev[1024][4];
void *nc__arena_alloc(nc_ctx *ctx, size_t bytes) { return bytes <= sizeof g_arena ? (void *)g_arena : 0; }
void nc__upload(nc_ctx *ctx, void *dst, const void *src, size_t bytes) { memcpy(g_dev, src, bytes); }

static void steps(uint64_t *s, long n) { for (long i = 0; i < n; i++) step(s); }

int main(void) {
    const int64_t count = 16384; /* runs of 64: 2^20 draws */
    const uint64_t *q = nc__rng_run_polys(count);
    if (!q || !g_charp_ok) { printf("FAIL table\n"); return 1; }
    /* P has degree 256 with a non-zero constant term (T is invertible) */
    if (!(g_charp[0] & 1u)) { printf("FAIL constant term\n"); return 1; }
    const long ks[] = {0, 1, 2, 63, 64, 1000, 16383};
    for (unsigned t = 0; t < sizeof ks / sizeof ks[0]; t++) {
        const long k = ks[t];
        uint64_t v[4] = {0x0123456789ABCDEFull, 42, 7, 0xFFFFFFFF00000000ull}, a[4], s[4];
        memcpy(s, v, sizeof s);
        poly_apply(q + 4 * k, v, a);
        steps(s, 64 * k);
        if (memcmp(a, s, sizeof a)) { printf("FAIL jump %ld\n", k); return 1; }
        /* four-word split: sum_j r_j(T) (T^(64 j) v) */
        uint64_t acc[4] = {0, 0, 0, 0}, b[4];
        memcpy(b, v, sizeof b);
        for (int j = 0; j < 4; j++) {
            uint64_t st[4], part[4] = {0, 0, 0, 0};
            memcpy(st, b, sizeof st);
            for (int i = 0; i < 64; i++) {
                if ((q[4 * k + j] >> i) & 1u) for (int e = 0; e < 4; e++) part[e] ^= st[e];
                step(st);
            }
            for (int e = 0; e < 4; e++) acc[e] ^= part[e];
            steps(b, 64);
        }
        if (memcmp(acc, s, sizeof acc)) { printf("FAIL split %ld\n", k); return 1; }
        /* the host-built window tables (nc__rng_dropout_tabs) evaluated as the kernel does */
        static nc_ctx ctx;
        memcpy(ctx.rng, v, sizeof v);
        if (nc__rng_dropout_tabs(&ctx) != (const void *)g_arena) { printf("FAIL tabs\n"); return 1; }
        uint64_t w4[4] = {0, 0, 0, 0};
        for (int j = 0; j < 4; j++)
            for (int nn = 0; nn < 16; nn++) {
                const uint64_t *e = g_dev[j * 256 + nn * 16 + ((q[4 * k + j] >> (4 * nn)) & 15)];
                for (int q2 = 0; q2 < 4; q2++) w4[q2] ^= e[q2];
            }
        if (memcmp(w4, s, sizeof w4)) { printf("FAIL windows %ld\n", k); return 1; }
    }
    printf("OK\n");
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_run_polynomials_match_sequential_stepping(tmp_path):
    src = tmp_path / "rng_jumps.c"
    src.write_text(HARNESS)
    exe = tmp_path / "rng_jumps"
    csrc = REPO / "newch_b200" / "csrc"
    subprocess.run(["gcc", "-O2", "-std=c11", "-D_GNU_SOURCE", f"-I{csrc}", "-I/usr/local/cuda/include",
                    str(src), "-o", str(exe), "-lpthread", "-lm"], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "OK", out.stdout + out.stderr
