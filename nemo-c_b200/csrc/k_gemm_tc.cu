// Tensor-core (tcgen05 / TMEM / TMA) GEMM for many rows. Placeholder until the sm_100a tiles land:
// every caller currently routes fp32 activations to the CUDA-core kernels in k_gemm.cu.
#include "common.cuh"

int nb_gemm_tc_supported(const nemo_gemm_args_t *a) { (void)a; return 0; }
int nb_gemm_tc(const nemo_gemm_args_t *a, void *stream) {
    (void)a; (void)stream;
    return nb_set_error("nemo_gemm: tensor-core path not available in this build");
}
