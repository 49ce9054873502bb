// Error reporting and launch accounting shared by every C-ABI entry point.
#include <atomic>
#include <mutex>
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

static thread_local int g_counting = 1;
// While a stream is being captured into a CUDA graph, launches are recorded, not executed: the
// engine turns counting off and adds the graph's kernel nodes each time it launches the graph.
extern "C" void nb_set_launch_counting(int on) { g_counting = on; }

extern "C" int nb_pdl_enabled(void) {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("NEMO_PDL");
        on = !(v && !strcmp(v, "0"));
    }
    return on;
}

int nb_check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return nb_set_error("%s: %s", what, cudaGetErrorString(e));
    if (g_counting) nb_count_launches(1);
    return 0;
}

// Number of kernel nodes in a graph (launch accounting of graph replays).
extern "C" uint64_t nb_graph_kernel_nodes(cudaGraph_t g) {
    size_t n = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || n == 0) return 0;
    cudaGraphNode_t *nodes = new cudaGraphNode_t[n];
    uint64_t k = 0;
    if (cudaGraphGetNodes(g, nodes, &n) == cudaSuccess)
        for (size_t i = 0; i < n; ++i) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
        }
    delete[] nodes;
    return k;
}

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the current device. The
// attribute belongs to the device, so the largest value set so far is kept per (kernel, device),
// under a lock: a second device, or a thread on another device, sets its own.
extern "C" int nb_smem_attr(const void *func, size_t bytes) {
    if (bytes <= 48 * 1024) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nb_set_error("no current CUDA device");
    struct Entry { const void *func; int dev; size_t bytes; };
    static Entry table[256];
    static int used = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int i = 0;
    while (i < used && !(table[i].func == func && table[i].dev == dev)) ++i;
    if (i < used && table[i].bytes >= bytes) return 0;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return nb_set_error("%zu bytes of dynamic shared memory unavailable: %s", bytes, cudaGetErrorString(cudaGetLastError()));
    if (i == used) {
        if (used == 256) return 0;  // full: the attribute is set, only the memo is skipped
        table[used++] = Entry{func, dev, bytes};
    } else {
        table[i].bytes = bytes;
    }
    return 0;
}
