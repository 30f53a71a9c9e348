// Instantiation of gemv_kernel for one activation-row count (GEMV_M), over
// the (prologue, epilogue) pairs the engine and the op surface use.
#include "ops.cuh"

#ifndef GEMV_M
#error "define GEMV_M"
#endif

#define SKB_CAT2(a, b) a##b
#define SKB_CAT(a, b) SKB_CAT2(a, b)

namespace skb {

template <int KV4, int XMV, int EMV>
static cudaError_t gemv_go(const GemvArgs& a, int grid, cudaStream_t s, bool pdl) {
    auto kern = gemv_kernel<GEMV_M, KV4, XMV, EMV>;
    if (grid <= 0)  // prepare only
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_MAX);
    const int G = gemv_grid(a.N, a.K, EMV, grid, GemvShape<GEMV_M, KV4>::RC);
    return launch(kern, dim3(G), dim3(GEMV_THREADS), gemv_smem_bytes(a.N, a.K, EMV, G), s, pdl, a);
}

template <int KV4>
static cudaError_t gemv_dispatch_em(const GemvArgs& a, int XM, int EM, int grid, cudaStream_t s, bool pdl) {
#define SKB_CASE(XMV, EMV)                                                                       \
    if (XM == XMV && EM == EMV) return gemv_go<KV4, XMV, EMV>(a, grid, s, pdl);
    SKB_CASE(X_PLAIN, E_STORE)
    SKB_CASE(X_PLAIN, E_RESID)
    SKB_CASE(X_PLAIN, E_BIAS)
    SKB_CASE(X_PLAIN, E_SWIGLU)
    SKB_CASE(X_RMSNORM, E_STORE)
    SKB_CASE(X_RMSNORM, E_SWIGLU)
    SKB_CASE(X_RMSNORM, E_BIAS)
    SKB_CASE(X_ADD_RMSNORM, E_SWIGLU)
    SKB_CASE(X_NORM_ADD_NORM, E_SWIGLU)
#undef SKB_CASE
    return cudaErrorInvalidValue;
}

cudaError_t SKB_CAT(gemv_prepare_m, GEMV_M)() {
    GemvArgs a = {};
    const int pairs[9][2] = {{X_PLAIN, E_STORE}, {X_PLAIN, E_RESID}, {X_PLAIN, E_BIAS}, {X_PLAIN, E_SWIGLU},
                             {X_RMSNORM, E_STORE}, {X_RMSNORM, E_SWIGLU}, {X_RMSNORM, E_BIAS},
                             {X_ADD_RMSNORM, E_SWIGLU}, {X_NORM_ADD_NORM, E_SWIGLU}};
    for (int kv4 = 1; kv4 <= 4; ++kv4)
        for (auto& p : pairs) {
            cudaError_t e = SKB_CAT(gemv_launch_m, GEMV_M)(a, kv4, p[0], p[1], 0, nullptr, false);
            if (e != cudaSuccess) return e;
        }
    return cudaSuccess;
}

cudaError_t SKB_CAT(gemv_launch_m, GEMV_M)(const GemvArgs& a, int KV4, int XM, int EM, int grid,
                                           cudaStream_t s, bool pdl) {
    switch (KV4) {
        case 1: return gemv_dispatch_em<1>(a, XM, EM, grid, s, pdl);
        case 2: return gemv_dispatch_em<2>(a, XM, EM, grid, s, pdl);
        case 3: return gemv_dispatch_em<3>(a, XM, EM, grid, s, pdl);
        case 4: return gemv_dispatch_em<4>(a, XM, EM, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace skb
