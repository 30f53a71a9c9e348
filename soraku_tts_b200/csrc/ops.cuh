// Internal declarations shared by the translation units of libsoraku_b200.so.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace skb {

int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
bool aligned16(const void* p);

struct NormRowsArgs {
    const float* x;
    int ldx;
    const float* x2;
    int ldx2, x2_div;
    const float* nw;
    float eps;
    const float* nw2;
    float eps2;
    float* xn;    // [rows][D]
    float* xout;  // optional copy of xn
    float* hout;  // optional inner norm (mode 3)
    int D, mode;  // mode 1 rmsnorm, 3 norm-add-norm
    unsigned long long* ts;  // optional debug timeline (kernel stamps [0..3])
};
int norm_rows(const NormRowsArgs& a, int rows, cudaStream_t s, bool pdl);
cudaError_t advance_launch(int* cnt, int n, cudaStream_t s, bool pdl);
int rmsnorm_rows(const float* x, const float* x2, const float* w, float* out, int B, int D,
                 float eps, cudaStream_t s, bool pdl);
int cfg_sample(const float* logits, int rows_per_req, int n_req, int V,
               const skb_sample_params* params, int bos, int pad, int eos, int64_t* codes,
               float* uniforms, cudaStream_t s, bool pdl);
GemvArgs gemv_args_plain(const float* x, int ldx, int N, int K);

struct RgPlan;
cudaError_t gemv_launch_m1(const GemvArgs& a, int KQ, int XM, int EM, const RgPlan& p, cudaStream_t s, bool pdl);
cudaError_t gemv_launch_m2(const GemvArgs& a, int KQ, int XM, int EM, const RgPlan& p, cudaStream_t s, bool pdl);
cudaError_t gemv_launch_m4(const GemvArgs& a, int KQ, int XM, int EM, const RgPlan& p, cudaStream_t s, bool pdl);
cudaError_t gemv_prepare_m1();
cudaError_t gemv_prepare_m2();
cudaError_t gemv_prepare_m4();

}  // namespace skb
