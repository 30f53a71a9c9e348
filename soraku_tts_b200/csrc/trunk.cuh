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
    int nmax;  // score slots per split (dynamic smem n_rep * nmax floats)
    float scale;
    float* part;    // [R][KVH][S][n_rep][hd + 2]
    int* counters;  // [R][KVH]
    float* out;     // [R][H*hd]
    int* err;
    PrefetchList pf;
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
    int mode;  // 0 store, 1 resid, 3 swiglu
};

}  // namespace skb
