// Error reporting and launch accounting shared by every C-ABI entry point.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include "common.cuh"

static thread_local char g_err[1024];
static std::atomic<uint64_t> g_launches{0};

extern "C" int nb_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return -1;
}
extern "C" const char *nemo_gpu_last_error(void) { return g_err; }
extern "C" void nb_count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
extern "C" uint64_t nemo_gpu_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int nb_check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return nb_set_error("%s: %s", what, cudaGetErrorString(e));
    nb_count_launches(1);
    return 0;
}
