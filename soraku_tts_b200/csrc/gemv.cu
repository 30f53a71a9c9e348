// Host dispatch of the decode GEMV over the activation-row count.
#include "ops.cuh"
#include "rgemv.cuh"

namespace skb {

static bool aligned_rows(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t gemv_launch(const GemvArgs& a, int M, int XM, int EM, int grid, cudaStream_t stream, bool pdl) {
    static bool prepared = false;
    if (!prepared) {
        const cudaError_t e = gemv_prepare_all();
        if (e != cudaSuccess) return e;
        prepared = true;
    }
    const RgPlan p = rgemv_plan(a.N, a.K, M, EM, grid);
    if (p.slots == 0 || (EM == E_SWIGLU && (a.N & 1)) || !aligned_rows(a.w0) || !aligned_rows(a.w1) ||
        !aligned_rows(a.w2))
        return cudaErrorInvalidValue;
    switch (M) {
        case 1: return gemv_launch_m1(a, p.kq, XM, EM, p, stream, pdl);
        case 2: return gemv_launch_m2(a, p.kq, XM, EM, p, stream, pdl);
        case 4: return gemv_launch_m4(a, p.kq, XM, EM, p, stream, pdl);
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
