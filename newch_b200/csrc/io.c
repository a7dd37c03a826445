/* Named-tensor files in newch's NCW1 format (newch docs/FORMAT.md; reader and writer in
 * engine/src/core/io.c:52-167): magic "NCW1", u32 version 1, u32 count, then per entry u32 name
 * length, name bytes, u32 dtype, u32 ndim, i64 shape[ndim], u64 byte count, row-major data; all
 * little-endian. Files are interchangeable with newch's. Device data passes through a host buffer.
 */
#define _FILE_OFFSET_BITS 64
#define _POSIX_C_SOURCE 200809L
#include "nc_internal.h"

#include <stdio.h>
#include <stdlib.h>

#define NCW_MAGIC "NCW1"
#define NCW_VERSION 1u
#define NCW_MAX_NAME 4096

static int put(FILE *f, const void *p, size_t n) { return fwrite(p, 1, n, f) == n; }
static int get(FILE *f, void *p, size_t n) { return fread(p, 1, n, f) == n; }

nc_status nc_save(nc_ctx *ctx, const char *path, int n, const char *const *names, nc_tensor *const *tensors) {
    if (ctx->status != NC_OK) return ctx->status;
    for (int i = 0; i < n; i++) {
        if (!tensors[i] || !names[i]) {
            nc__error(ctx, NC_ERR_ARG, "nc_save: entry %d has a NULL name or tensor", i);
            return ctx->status;
        }
    }
    FILE *f = fopen(path, "wb");
    if (!f) {
        nc__error(ctx, NC_ERR_ARG, "nc_save: cannot open '%s' for writing", path);
        return ctx->status;
    }
    uint32_t version = NCW_VERSION, count = (uint32_t)n;
    int ok = put(f, NCW_MAGIC, 4) && put(f, &version, 4) && put(f, &count, 4);
    for (int i = 0; ok && i < n; i++) {
        const nc_tensor *t = tensors[i];
        uint32_t len = (uint32_t)strlen(names[i]), dt = (uint32_t)t->dtype, nd = (uint32_t)t->ndim;
        uint64_t bytes = (uint64_t)nc_numel(t) * nc__dtype_size(t->dtype);
        ok = put(f, &len, 4) && put(f, names[i], len) && put(f, &dt, 4) && put(f, &nd, 4) &&
             put(f, t->shape, sizeof(int64_t) * nd) && put(f, &bytes, 8);
        if (!ok || !bytes) continue;
        void *tmp = malloc((size_t)bytes);
        ok = tmp && nc_copy_to(t, tmp, (size_t)bytes) && put(f, tmp, (size_t)bytes);
        free(tmp);
    }
    if (fclose(f) != 0) ok = 0;
    if (!ok) nc__error(ctx, NC_ERR_ARG, "nc_save: write to '%s' failed", path);
    return ctx->status;
}

nc_status nc_load(nc_ctx *ctx, const char *path, int n, const char *const *names, nc_tensor *const *tensors) {
    if (ctx->status != NC_OK) return ctx->status;
    FILE *f = fopen(path, "rb");
    if (!f) {
        nc__error(ctx, NC_ERR_ARG, "nc_load: cannot open '%s'", path);
        return ctx->status;
    }
    unsigned char *found = (unsigned char *)calloc((size_t)(n ? n : 1), 1);
    char *name = (char *)malloc(NCW_MAX_NAME + 1);
    void *buf = NULL;
    char magic[4];
    uint32_t version = 0, count = 0;
    if (!found || !name) {
        nc__error(ctx, NC_ERR_OOM, "nc_load: out of memory");
        goto done;
    }
    if (!get(f, magic, 4) || memcmp(magic, NCW_MAGIC, 4) != 0 || !get(f, &version, 4) || !get(f, &count, 4)) {
        nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' is not an NCW1 tensor file", path);
        goto done;
    }
    if (version != NCW_VERSION) {
        nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' has unsupported version %u", path, version);
        goto done;
    }
    for (uint32_t e = 0; e < count; e++) {
        uint32_t len, dt, nd;
        int64_t shape[NC_MAX_DIMS];
        uint64_t bytes;
        if (!get(f, &len, 4) || len > NCW_MAX_NAME || !get(f, name, len) || !get(f, &dt, 4) || !get(f, &nd, 4) ||
            nd > NC_MAX_DIMS || !get(f, shape, sizeof(int64_t) * nd) || !get(f, &bytes, 8)) {
            nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' is truncated or corrupt", path);
            goto done;
        }
        name[len] = '\0';
        int idx = -1;
        for (int i = 0; i < n; i++)
            if (!found[i] && strcmp(names[i], name) == 0) idx = i;
        if (idx < 0) {
            if (fseeko(f, (off_t)bytes, SEEK_CUR) != 0) {
                nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' is truncated", path);
                goto done;
            }
            continue;
        }
        nc_tensor *t = tensors[idx];
        int same = t->dtype == (nc_dtype)dt && t->ndim == (int)nd;
        for (uint32_t d = 0; same && d < nd; d++) same = t->shape[d] == shape[d];
        if (!same) {
            char want[96], got[96];
            nc__error(ctx, NC_ERR_SHAPE, "nc_load: '%s' is %s %s in the file but %s %s in the model", name,
                      nc__dtype_name((nc_dtype)dt), nc__shape_str((int)nd, shape, got, sizeof got),
                      nc__dtype_name(t->dtype), nc__shape_str(t->ndim, t->shape, want, sizeof want));
            goto done;
        }
        if (bytes != (uint64_t)nc_numel(t) * nc__dtype_size(t->dtype)) {
            nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' in '%s' is corrupt (%llu data bytes for %s)", name, path,
                      (unsigned long long)bytes, nc__dtype_name(t->dtype));
            goto done;
        }
        free(buf);
        buf = malloc((size_t)(bytes ? bytes : 1));
        if (!buf || !nc_is_contiguous(t) || !get(f, buf, (size_t)bytes) ||
            (bytes && !nc_copy_from(t, buf, (size_t)bytes))) {
            nc__error(ctx, NC_ERR_ARG, "nc_load: cannot read '%s' (truncated file or non-contiguous tensor)", name);
            goto done;
        }
        found[idx] = 1;
    }
    for (int i = 0; i < n; i++) {
        if (!found[i]) {
            nc__error(ctx, NC_ERR_ARG, "nc_load: '%s' not found in '%s'", names[i], path);
            break;
        }
    }
done:
    free(buf);
    free(found);
    free(name);
    fclose(f);
    return ctx->status;
}
