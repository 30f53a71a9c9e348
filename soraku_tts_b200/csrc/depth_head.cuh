// Persistent depth head for one CFG request (depth_head.cu): the 16 depth
// steps of a frame as one cooperative launch, one CTA per SM.
#pragma once

#include "engine_types.cuh"

namespace skb {

struct DepthArgs {
    int V, Q;  // audio vocabulary, codebooks (model width 1024, depth inner size 2048)
    float rms_eps, depth_eps, scale;
    const float* final_norm;  // trunk final norm [1024]
    const float* norm_in;     // depth_head.norm_in [1024]
    const float* norm_out;    // depth_head.norm_out [1024]
    const float* wg;          // [2048][1024]
    const float* wu;          // [2048][1024]
    const float* wd;          // [1024][2048]
    const float* table;       // [Q][V][1024]
    const float* bias;        // [Q][V]
    float* x;       // [2][1024] trunk output in; the frame embedding out
    float* act;     // [2][2048] scratch
    float* y;       // [2][1024] scratch
    float* hidden;  // [2][1024] the final-normed trunk output (written by CTA 0)
    float* logits;  // [2][V], or one [2][V] buffer per codebook every logits_q_stride floats
    int logits_q_stride;
    ReqState* st;
    const int* host_flag;
    int64_t* cur_codes;  // [Q]
    int64_t* hist;       // [max_frames][Q]
    int max_frames;
    int bos, pad, eos;
    unsigned* bar;  // grid barrier word (sense-reversing, zero at creation)
    int* abort;     // raised by the CTA whose wait timed out
    int* err;       // [8]: err[3] a wait of this kernel timed out
    unsigned long long* ts;  // optional debug timeline [4 Q][2]: CTA 0's phase release / end
};

// True when this device and model can run the persistent depth head (model
// width 1024, inner 2048, vocabulary <= 2304, enough SMs, cooperative launch).
bool depth_head_supported(int D, int I, int V, int Q, int nsm, int device);
cudaError_t depth_head_prepare();
// One launch: `grid` CTAs (one per SM), cooperative.
cudaError_t depth_head_launch(const DepthArgs& a, int grid, cudaStream_t s);
int depth_head_phases(int Q);

}  // namespace skb
