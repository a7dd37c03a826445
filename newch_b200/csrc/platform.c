/* Host CPU facts for nc_cpu (newch engine/src/runtime/cpu_features.c reports the same fields).
 * The B200 engine computes on the GPU; these only describe the host that drives it. */
#include "nc_internal.h"

#include <unistd.h>

void nc__detect_cpu(nc_cpu_info *info) {
    memset(info, 0, sizeof *info);
#if defined(__x86_64__)
    info->arch = "x86_64";
    __builtin_cpu_init();
    info->has_avx2 = __builtin_cpu_supports("avx2") ? 1 : 0;
    info->has_fma = __builtin_cpu_supports("fma") ? 1 : 0;
#elif defined(__aarch64__)
    info->arch = "aarch64";
    info->has_neon = 1;
#else
    info->arch = "unknown";
#endif
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    info->n_cores = n > 0 ? (int)n : 1;
    info->n_big_cores = info->n_cores;
}
