// Instantiation of the ring-streamed decode GEMV (rgemv_kernel) for one
// activation-row count (GEMV_M), over the inner sizes K <= 1024, 2048, 3072
// and the (prologue, epilogue) pairs the engine and the op surface use.
#include "ops.cuh"
#include "rgemv.cuh"

#ifndef GEMV_M
#error "define GEMV_M"
#endif

#define SKB_CAT2(a, b) a##b
#define SKB_CAT(a, b) SKB_CAT2(a, b)

namespace skb {

template <int KQ, int XMV, int EMV>
static cudaError_t gemv_go(const GemvArgs& a, const RgPlan& p, cudaStream_t s, bool pdl) {
    constexpr bool XR = (KQ == 8 && GEMV_M <= 2);
    constexpr bool KS_OK = (KQ > 8 && EMV != E_SWIGLU && GEMV_M * RG_KS_UNITS <= 32);
    auto kern = rgemv_kernel<GEMV_M, KQ, XMV, EMV, XR, false>;
    if constexpr (KS_OK) {
        auto kks = rgemv_kernel<GEMV_M, KQ, XMV, EMV, false, true>;
        if (p.grid <= 0) {  // prepare only
            const cudaError_t e = set_smem_attrs(kks, RG_SMEM_MAX);
            if (e != cudaSuccess) return e;
        } else if (p.ks) {
            return launch(kks, dim3(p.grid), dim3(RG_THREADS), p.smem, s, pdl, a, p.slots);
        }
    }
    if (p.grid <= 0) return set_smem_attrs(kern, RG_SMEM_MAX);
    if (p.ks) return cudaErrorInvalidValue;
    return launch(kern, dim3(p.grid), dim3(RG_THREADS), p.smem, s, pdl, a, p.slots);
}

template <int KQ>
static cudaError_t gemv_dispatch_em(const GemvArgs& a, int XM, int EM, const RgPlan& p, cudaStream_t s,
                                    bool pdl) {
#define SKB_CASE(XMV, EMV) \
    if (XM == XMV && EM == EMV) return gemv_go<KQ, XMV, EMV>(a, p, s, pdl);
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

cudaError_t SKB_CAT(gemv_launch_m, GEMV_M)(const GemvArgs& a, int KQ, int XM, int EM, const RgPlan& p,
                                           cudaStream_t s, bool pdl) {
    switch (KQ) {
        case 8: return gemv_dispatch_em<8>(a, XM, EM, p, s, pdl);
        case 16: return gemv_dispatch_em<16>(a, XM, EM, p, s, pdl);
        case 24: return gemv_dispatch_em<24>(a, XM, EM, p, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t SKB_CAT(gemv_prepare_m, GEMV_M)() {
    GemvArgs a = {};
    RgPlan p;  // grid 0: set attributes only
    const int pairs[9][2] = {{X_PLAIN, E_STORE}, {X_PLAIN, E_RESID}, {X_PLAIN, E_BIAS}, {X_PLAIN, E_SWIGLU},
                             {X_RMSNORM, E_STORE}, {X_RMSNORM, E_SWIGLU}, {X_RMSNORM, E_BIAS},
                             {X_ADD_RMSNORM, E_SWIGLU}, {X_NORM_ADD_NORM, E_SWIGLU}};
    for (int kq : {8, 16, 24})
        for (auto& pr : pairs) {
            cudaError_t e = SKB_CAT(gemv_launch_m, GEMV_M)(a, kq, pr[0], pr[1], p, nullptr, false);
            if (e != cudaSuccess) return e;
        }
    return cudaSuccess;
}

}  // namespace skb
