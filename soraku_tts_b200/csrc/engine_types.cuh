// Engine state: per-request sampling state and the depth-sampler step.
#pragma once

#include "common.cuh"
#include "sampler.cuh"

namespace skb {

struct ReqState {
    float cfg, temp, temp_q0, top_p, top_p_q0;
    int top_k, top_k_q0, min_new_frames, eos_rule;
    int frame;  // frames completed (advanced by the q = Q-1 sampler)
    int done;   // q0 drew EOS at least once
    unsigned stream;  // Philox counter word 1: the request's random stream (default: its slot)
    unsigned long long seed;
};

struct DepthSampleArgs {
    const float* logits;  // [R][V]
    int rows_per_req, V, q, Q, D;
    ReqState* st;
    const int* host_flag;
    const float* table;
    float scale;
    float* prefix;  // [n_req][D]
    float* x;       // [R][D]
    int64_t* cur_codes;  // [n_req][Q]
    int64_t* hist;       // [n_req][max_frames][Q]
    int max_frames;
    int bos, pad, eos;
    // Optional (batched rows, codebooks before the last): the next depth
    // step's input rows, a = norm_in(final_norm(x) + prefix) with the updated
    // prefix, written here instead of by a row-norm launch: xn and xout get a,
    // hout the final-normed x (null: not done)
    const float* fn_w;  // final norm weight [D]
    float fn_eps;
    const float* ni_w;  // depth norm_in weight [D]
    float ni_eps;
    float *xn, *xout, *hout;  // [R][D]
    PrefetchList pf;
    unsigned long long* ts;  // optional debug timeline [4]
};

// The sampling job of request r for codebook a.q.  It reads only the
// request's state and the host EOS flag, which no kernel of the current
// frame writes before the sampler, so a kernel may build it before its
// programmatic-dependent-launch wait.
__device__ __forceinline__ SampleJob depth_sample_job(const DepthSampleArgs& a, int r, int* frame_out) {
    const ReqState* st = a.st + r;
    const int frame = __ldcg(&st->frame);
    const bool q0 = a.q == 0;
    SampleJob J;
    J.cond = a.logits + (size_t)r * a.rows_per_req * a.V;
    J.uncond = a.rows_per_req > 1 ? J.cond + a.V : nullptr;
    J.V = a.V;
    J.cfg_scale = st->cfg;
    J.temperature = q0 ? st->temp_q0 : st->temp;
    J.top_k = q0 ? st->top_k_q0 : st->top_k;
    J.top_p = q0 ? st->top_p_q0 : st->top_p;
    J.mask_eos = !q0 ? 1 : (st->eos_rule == 0 ? (__ldcg(a.host_flag) != 0) : (frame < st->min_new_frames));
    J.bos = a.bos;
    J.pad = a.pad;
    J.eos = a.eos;
    J.u = philox_uniform(st->seed, st->stream, (uint32_t)frame, (uint32_t)a.q);
    J.ts = a.ts;
    *frame_out = frame;
    return J;
}

// Block sum of one float per thread (256 threads); red: 8 floats of shared memory.
template <class Sync>
__device__ __forceinline__ float depth_block_sum(float v, float* red) {
    v = warp_sum(v);
    Sync::sync();  // red is free (its last readers are done)
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    Sync::sync();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    return t;
}

// The next depth step's input rows of request r (its rows_per_req rows):
// h = fn_w * (x * inv_rms(x)), v = h + prefix, a = ni_w * (v * inv_rms(v)),
// the operations and order of the row-norm kernel they replace.  pv: this
// thread's prefix values (columns tid + 256 j).
template <class Sync>
__device__ void depth_next_rows(const DepthSampleArgs& a, int r, const float (&pv)[4], float* red) {
    const int tid = threadIdx.x;
    for (int rr = 0; rr < a.rows_per_req; ++rr) {
        const size_t row = (size_t)r * a.rows_per_req + rr;
        float v[4];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + SAMPLER_THREADS * j;
            v[j] = i < a.D ? __ldcg(a.x + row * a.D + i) : 0.f;
            ss += v[j] * v[j];
        }
        const float inv1 = rsqrtf(depth_block_sum<Sync>(ss, red) / (float)a.D + a.fn_eps);
        ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + SAMPLER_THREADS * j;
            if (i < a.D) {
                const float h = a.fn_w[i] * (v[j] * inv1);
                if (a.hout) a.hout[row * a.D + i] = h;
                v[j] = h + pv[j];
            }
            ss += v[j] * v[j];
        }
        const float inv2 = rsqrtf(depth_block_sum<Sync>(ss, red) / (float)a.D + a.ni_eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + SAMPLER_THREADS * j;
            if (i < a.D) {
                const float o = a.ni_w[i] * (v[j] * inv2);
                a.xn[row * a.D + i] = o;
                if (a.xout) a.xout[row * a.D + i] = o;
            }
        }
    }
}

// One request's sampling step for codebook a.q (job J from depth_sample_job)
// and its epilogue: the code goes to the current-frame and history buffers,
// the prefix grows by table[q][code] * scale, and after the last codebook the
// frame embedding (sum over q in order, then * scale) becomes both CFG rows'
// residual stream, the prefix is cleared and the request's frame counter
// advances.  Threads 0..255 take part.  codes_s: 32 ints of shared memory.
template <class Sync, int VMAX>
__device__ void depth_sample_body(const DepthSampleArgs& a, int r, const SampleJob& J, int frame,
                                  unsigned char* smem, int* codes_s) {
    const int tid = threadIdx.x;
    ReqState* st = a.st + r;
    const bool q0 = a.q == 0;
    if (tid == 0 && a.ts) stamp_max(a.ts + 4);
    const int code = sample_one<Sync, VMAX>(J, smem);
    if (tid == 0 && a.ts) stamp_max(a.ts + 11);
    if (tid == 0) {
        a.cur_codes[(size_t)r * a.Q + a.q] = code;
        if (frame < a.max_frames) a.hist[((size_t)r * a.max_frames + frame) * a.Q + a.q] = code;
        if (q0 && code == a.eos) st->done = 1;
    }
    float* pr = a.prefix + (size_t)r * a.D;
    if (a.q < a.Q - 1) {
        const float* trow = a.table + ((size_t)a.q * a.V + code) * a.D;
        if (a.xn == nullptr) {
            for (int i = tid; i < a.D; i += SAMPLER_THREADS) pr[i] = __ldcg(pr + i) + trow[i] * a.scale;
        } else {
            // the updated prefix stays in registers for the next step's rows
            constexpr int PT = 4;  // D / 256 (D <= 1024)
            float pv[PT];
#pragma unroll
            for (int j = 0; j < PT; ++j) {
                const int i = tid + SAMPLER_THREADS * j;
                pv[j] = 0.f;
                if (i < a.D) {
                    pv[j] = __ldcg(pr + i) + trow[i] * a.scale;
                    pr[i] = pv[j];
                }
            }
            depth_next_rows<Sync>(a, r, pv, reinterpret_cast<float*>(smem));
        }
    } else {
        if (tid < a.Q) codes_s[tid] = (tid == a.q) ? code : (int)__ldcg(a.cur_codes + (size_t)r * a.Q + tid);
        Sync::sync();
        for (int i = tid; i < a.D; i += SAMPLER_THREADS) {
            // all codebooks' rows are requested before the in-order sum
            float v[32];
#pragma unroll
            for (int qq = 0; qq < 32; ++qq) {
                int c = qq < a.Q ? codes_s[qq] : 0;
                if (c < 0 || c >= a.V) c = 0;
                v[qq] = qq < a.Q ? a.table[((size_t)qq * a.V + c) * a.D + i] : 0.f;
            }
            float acc = v[0];
#pragma unroll
            for (int qq = 1; qq < 32; ++qq)
                if (qq < a.Q) acc = acc + v[qq];
            acc = acc * a.scale;
            for (int rr = 0; rr < a.rows_per_req; ++rr) a.x[((size_t)r * a.rows_per_req + rr) * a.D + i] = acc;
            pr[i] = 0.f;
        }
        if (tid == 0) st->frame = frame + 1;
    }
}


}  // namespace skb
