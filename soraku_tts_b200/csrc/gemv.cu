// Host dispatch of the decode GEMV over the activation-row count.
#include "ops.cuh"

namespace skb {

cudaError_t gemv_launch(const GemvArgs& a, int M, int XM, int EM, int grid, cudaStream_t stream,
                        bool pdl) {
    static bool prepared = false;
    if (!prepared) {
        const cudaError_t e = gemv_prepare_all();
        if (e != cudaSuccess) return e;
        prepared = true;
    }
    const int kv4 = ((a.K >> 2) + GEMV_THREADS - 1) / GEMV_THREADS;
    if (kv4 < 1 || kv4 > 4 || (a.K & 3) != 0) return cudaErrorInvalidValue;
    switch (M) {
        case 1: return gemv_launch_m1(a, kv4, XM, EM, grid, stream, pdl);
        case 2: return gemv_launch_m2(a, kv4, XM, EM, grid, stream, pdl);
        case 4: return gemv_launch_m4(a, kv4, XM, EM, grid, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemv_prepare_all() {
    cudaError_t e = gemv_prepare_m1();
    if (e == cudaSuccess) e = gemv_prepare_m2();
    if (e == cudaSuccess) e = gemv_prepare_m4();
    return e;
}

}  // namespace skb
