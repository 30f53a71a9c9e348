// Qwen3 trunk kernels: decode attention over the paged FP32 KV cache and the
// prefill path.  Arithmetic follows transformers' Qwen3 decoder
// (modeling_qwen3.py: RMSNorm :59-64, q_norm/k_norm :248-249, RoPE
// :130-181, GQA attention :184-219 with scaling head_dim**-0.5 :232).
#pragma once

#include "common.cuh"

namespace skb {

// KV pool: per layer [n_pages][2 (K, V)][KVH][page][head_dim] floats.
struct KVLayout {
    float* pool;
    const int* page_table;  // [rows][max_pages]
    int max_pages;
    int page_log2;
    int KVH;
    int hd;
    long long layer_floats;  // floats per layer
    int n_pages;             // pages per layer; table entries outside [0, n_pages) read page 0
    __device__ __forceinline__ float* at(int layer, int row, int pos, int kv, int g) const {
        int page = page_table[row * max_pages + (pos >> page_log2)];
        if ((unsigned)page >= (unsigned)n_pages) page = 0;
        const int slot = pos & ((1 << page_log2) - 1);
        return pool + layer * layer_floats +
               ((((long long)page * 2 + kv) * KVH + g) << page_log2) * hd + (long long)slot * hd;
    }
};

struct DecodeAttnArgs {
    const float* qkv;  // [R][ld_qkv]: q (H*hd) | k (KVH*hd) | v (KVH*hd)
    int ld_qkv;
    const float* qn;  // q_norm weight [hd]
    const float* kn;  // k_norm weight [hd]
    float eps;
    const float* rope_cos;  // [max_len][hd/2]
    const float* rope_sin;
    const int* pos;  // [R] position of the new token
    int max_len;
    KVLayout kv;
    int layer;
    int H, n_rep, S;
    int variant;  // cluster kernel: 0 by rows, 1 single-buffered (few groups), 2 double-buffered
    int nmax;  // score slots per split (dynamic smem n_rep * nmax floats)
    float scale;
    float* part;    // [R][KVH][S][n_rep][hd + 2]
    int* counters;  // [R][KVH]
    float* out;     // [R][H*hd]
    int* err;
    PrefetchList pf;
    unsigned long long* ts;  // optional debug timeline [4]
};

// prefill
struct PrefillTok {
    int row;   // CFG row
    int pos;   // logical position
    int kind;  // 0 text id, 1 audio frame, 2 speaker slot
    int val;   // text id or audio frame index
};

struct GemmArgs {
    const float* A;  // [T][K]
    int lda;
    const float* w0;
    const float* w1;
    const float* w2;
    int seg1, seg2, interleave;
    int N, K, T;
    float* out;
    int ldo;
    const float* resid;
    int ldr;
    const float* bias;  // [N] (mode 2)
    int mode;  // 0 store, 1 resid, 2 bias, 3 swiglu
    int* err;  // optional: set when a wait timed out (tensor-core GEMM)
    int splits;  // tensor-core GEMM: K splits per output tile (0 = chosen by occupancy)
    // kernel: 0 chooses by rows (the FFMA kernel for T <= 16 when it takes
    // the shape, else the tensor-core GEMM), 1 the tensor-core GEMM, 2 the
    // FFMA kernel (T <= 32)
    int variant;
    // debug timeline (null: off): [0..3] as for every kernel; tensor-core
    // GEMM: [4] latest / [8] earliest first stage at the MMA, [5] latest
    // all-MMAs-done, [6] latest result staged (after the cluster barrier),
    // [7] latest output stores issued; FFMA kernel: [4] latest first chunk
    // landed, [5] all chunks consumed, [6] partials reduced, [8 + c] / [12 +
    // c] chunk c (< 4) landed / consumed
    unsigned long long* ts;
};


// Shared memory of one decode-attention work item.
struct AttnSmem {
    __align__(16) float qs[2][128];
    __align__(16) float ks[128];
    __align__(16) float vs[128];
    __align__(16) float wo[8][2][128];
    float wm[8][2], wl[8][2];
    int last;
};

// q/k RMSNorm over one head (hd = 128, 4 elements per lane) then neox RoPE.
// Lane l holds elements [4l, 4l+4); its RoPE partner elements (+-64) live in
// lane l ^ 16.
__device__ __forceinline__ float4 norm_rope_head(float4 x, const float* w, float eps,
                                                 const float* cosr, const float* sinr, int lane,
                                                 bool do_norm, bool do_rope) {
    if (do_norm) {
        float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / 128.0f + eps);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + lane);
        x.x = wv.x * (x.x * inv);
        x.y = wv.y * (x.y * inv);
        x.z = wv.z * (x.z * inv);
        x.w = wv.w * (x.w * inv);
    }
    if (do_rope) {
        float4 o;
        o.x = __shfl_xor_sync(FULL, x.x, 16);
        o.y = __shfl_xor_sync(FULL, x.y, 16);
        o.z = __shfl_xor_sync(FULL, x.z, 16);
        o.w = __shfl_xor_sync(FULL, x.w, 16);
        const int i0 = (lane & 15) * 4;  // frequency index of element 0
        const float4 c = *reinterpret_cast<const float4*>(cosr + i0);
        const float4 s = *reinterpret_cast<const float4*>(sinr + i0);
        if (lane < 16) {  // first half: x*cos - x[i+64]*sin
            x.x = x.x * c.x - o.x * s.x;
            x.y = x.y * c.y - o.y * s.y;
            x.z = x.z * c.z - o.z * s.z;
            x.w = x.w * c.w - o.w * s.w;
        } else {  // second half: x*cos + x[i-64]*sin
            x.x = x.x * c.x + o.x * s.x;
            x.y = x.y * c.y + o.y * s.y;
            x.z = x.z * c.z + o.z * s.z;
            x.w = x.w * c.w + o.w * s.w;
        }
    }
    return x;
}

// grid (S, KVH, R), 256 threads.  CTA (s, g, r) owns positions
// [s*T/S, (s+1)*T/S) of row r's cache for kv head g (T = cached length + 1).
// Warp w takes positions pb+w, pb+w+8, ... in batches of 4: the K and V rows of
// a batch (512 B each, one float4 per lane) are loaded together, scores are
// warp-reduced, and an online softmax keeps (max, sum, o[h][lane*4..+4]) per
// warp.  The 8 warps merge through shared memory into the CTA's partial; the
// last CTA of each (row, kv head) -- an atomic ticket, no waiting -- merges the
// S partials in split order and writes the attention output.
constexpr int ATT_B = 4;

template <class Sync>
__device__ void decode_attn_item(const DecodeAttnArgs& a, int s, int g, int r, AttnSmem& sm) {
    float (&qs)[2][128] = sm.qs;
    float (&ks)[128] = sm.ks;
    float (&vs)[128] = sm.vs;
    float (&wo)[8][2][128] = sm.wo;
    float (&wm)[8][2] = sm.wm;
    float (&wl)[8][2] = sm.wl;
    int& sm_last = sm.last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    int p_new = __ldcg(a.pos + r);  // other CTAs advance positions: read through L2
    if (p_new < 0 || p_new >= a.max_len) {
        if (tid == 0 && a.err != nullptr) atomicExch(a.err, 1);
        p_new = p_new < 0 ? 0 : a.max_len - 1;
    }
    const int T = p_new + 1;
    const float* row = a.qkv + (size_t)r * a.ld_qkv;
    const float* cosr = a.rope_cos + (size_t)p_new * 64;
    const float* sinr = a.rope_sin + (size_t)p_new * 64;
    const int n_rep = a.n_rep;
    if (warp == 0) {
        float4 k = ld_cg4(reinterpret_cast<const float4*>(row + (a.H + g) * 128) + lane);
        k = norm_rope_head(k, a.kn, a.eps, cosr, sinr, lane, true, true);
        reinterpret_cast<float4*>(ks)[lane] = k;
    } else if (warp <= n_rep) {
        const int h = g * n_rep + (warp - 1);
        float4 q = ld_cg4(reinterpret_cast<const float4*>(row + h * 128) + lane);
        q = norm_rope_head(q, a.qn, a.eps, cosr, sinr, lane, true, true);
        q.x *= a.scale;
        q.y *= a.scale;
        q.z *= a.scale;
        q.w *= a.scale;
        reinterpret_cast<float4*>(qs[warp - 1])[lane] = q;
    } else if (warp == n_rep + 1) {
        const float4 v =
            ld_cg4(reinterpret_cast<const float4*>(row + (a.H + a.kv.KVH + g) * 128) + lane);
        reinterpret_cast<float4*>(vs)[lane] = v;
    }
    Sync::sync();

    const int pb = (int)((long long)s * T / a.S);
    const int pe = (int)((long long)(s + 1) * T / a.S);
    if (s == a.S - 1 && tid < 128) {
        a.kv.at(a.layer, r, p_new, 0, g)[tid] = ks[tid];
        a.kv.at(a.layer, r, p_new, 1, g)[tid] = vs[tid];
    }
    float4 q4[2];
    q4[0] = reinterpret_cast<const float4*>(qs[0])[lane];
    q4[1] = n_rep > 1 ? reinterpret_cast<const float4*>(qs[1])[lane] : q4[0];
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float4 o[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    // K/V rows of one batch of ATT_B positions (one float4 per lane each); the
    // next batch is loaded before the current one is consumed.
    auto load_batch = [&](int p0, float4 (&kb)[ATT_B], float4 (&vb)[ATT_B]) {
#pragma unroll
        for (int j = 0; j < ATT_B; ++j) {
            const int p = p0 + 8 * j;
            if (p < pe) {
                if (p == p_new) {
                    kb[j] = reinterpret_cast<const float4*>(ks)[lane];
                    vb[j] = reinterpret_cast<const float4*>(vs)[lane];
                } else {
                    kb[j] = ld_cg4(reinterpret_cast<const float4*>(a.kv.at(a.layer, r, p, 0, g)) + lane);
                    vb[j] = ld_cg4(reinterpret_cast<const float4*>(a.kv.at(a.layer, r, p, 1, g)) + lane);
                }
            } else {
                kb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                vb[j] = kb[j];
            }
        }
    };
    float4 kb[ATT_B], vb[ATT_B], kn[ATT_B], vn[ATT_B];
    if (pb + warp < pe) load_batch(pb + warp, kb, vb);
    for (int p0 = pb + warp; p0 < pe; p0 += 8 * ATT_B) {
        const bool more = p0 + 8 * ATT_B < pe;
        if (more) load_batch(p0 + 8 * ATT_B, kn, vn);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h >= n_rep) break;
            float sc[ATT_B];
#pragma unroll
            for (int j = 0; j < ATT_B; ++j) {
                float d = q4[h].x * kb[j].x + q4[h].y * kb[j].y + q4[h].z * kb[j].z + q4[h].w * kb[j].w;
                d = warp_sum(d);
                sc[j] = (p0 + 8 * j < pe) ? d : -INFINITY;
            }
            float mt = sc[0];
#pragma unroll
            for (int j = 1; j < ATT_B; ++j) mt = fmaxf(mt, sc[j]);
            const float mn = fmaxf(m[h], mt);
            const float corr = expf(m[h] - mn);
            float lsum = l[h] * corr;
            float4 acc = make_float4(o[h].x * corr, o[h].y * corr, o[h].z * corr, o[h].w * corr);
#pragma unroll
            for (int j = 0; j < ATT_B; ++j) {
                const float e = expf(sc[j] - mn);
                lsum += e;
                acc.x = fmaf(e, vb[j].x, acc.x);
                acc.y = fmaf(e, vb[j].y, acc.y);
                acc.z = fmaf(e, vb[j].z, acc.z);
                acc.w = fmaf(e, vb[j].w, acc.w);
            }
            m[h] = mn;
            l[h] = lsum;
            o[h] = acc;
        }
        if (more) {
#pragma unroll
            for (int j = 0; j < ATT_B; ++j) {
                kb[j] = kn[j];
                vb[j] = vn[j];
            }
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (h >= n_rep) break;
        reinterpret_cast<float4*>(wo[warp][h])[lane] = o[h];
        if (lane == 0) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
    }
    Sync::sync();
    const int hd2 = 128 + 2;
    float* part = a.part + ((((size_t)r * a.kv.KVH + g) * a.S + s) * n_rep) * hd2;
    if (tid < n_rep * 128) {
        const int h = tid >> 7, d = tid & 127;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w][h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const float c = expf(wm[w][h] - M);
                L = fmaf(wl[w][h], c, L);
                O = fmaf(wo[w][h][d], c, O);
            }
        }
        part[h * hd2 + d] = O;
        if (d == 0) {
            part[h * hd2 + 128] = M;
            part[h * hd2 + 129] = L;
        }
    }
    __threadfence();
    Sync::sync();
    if (tid == 0) sm_last = (atomicAdd(&a.counters[r * a.kv.KVH + g], 1) == a.S - 1) ? 1 : 0;
    Sync::sync();
    if (!sm_last) {
        Sync::sync();  // sm_last and the staging buffers are reused by the next item
        return;
    }
    __threadfence();
    // Merge the S split partials in split order.  The (max, sum) pairs are
    // staged in shared memory by parallel loads first, so the weighted sum over
    // the splits issues its partial-output loads independently of each other.
    {
        const float* base = a.part + ((((size_t)r * a.kv.KVH + g) * a.S) * n_rep) * hd2;
        float* sm_ml = &wo[0][0][0];  // reuse: [S][n_rep][2] (S * 4 floats <= 2048)
        for (int i = tid; i < a.S * n_rep; i += 256) {
            sm_ml[2 * i] = __ldcg(base + (size_t)i * hd2 + 128);
            sm_ml[2 * i + 1] = __ldcg(base + (size_t)i * hd2 + 129);
        }
        Sync::sync();
        if (tid < n_rep * 128) {
            const int h = tid >> 7, d = tid & 127;
            float M = -INFINITY;
            for (int j = 0; j < a.S; ++j) M = fmaxf(M, sm_ml[2 * (j * n_rep + h)]);
            float L = 0.f, O = 0.f;
#pragma unroll 8
            for (int j = 0; j < a.S; ++j) {
                const float mj = sm_ml[2 * (j * n_rep + h)];
                const float w = (mj == -INFINITY) ? 0.f : expf(mj - M);
                L = fmaf(sm_ml[2 * (j * n_rep + h) + 1], w, L);
                O = fmaf(__ldcg(base + ((size_t)j * n_rep + h) * hd2 + d), w, O);
            }
            a.out[(size_t)r * a.H * 128 + (g * n_rep + h) * 128 + d] = O / L;
        }
    }
    if (tid == 0) a.counters[r * a.kv.KVH + g] = 0;
    Sync::sync();
}


}  // namespace skb
