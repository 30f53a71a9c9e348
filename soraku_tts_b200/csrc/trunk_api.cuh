// Host launchers of trunk.cu.
#pragma once

#include "trunk.cuh"

namespace skb {

cudaError_t decode_attn_launch(const DecodeAttnArgs& a, int R, cudaStream_t s, bool pdl);
// Cluster variant (attn_cluster.cu): a.S = CTAs per (row, kv head), 1..8.
cudaError_t decode_attn_cluster_launch(const DecodeAttnArgs& a, int R, cudaStream_t s, bool pdl);
cudaError_t decode_attn_cluster_prepare();
cudaError_t tgemm_prepare();
int decode_attn_cluster_width(int groups);
cudaError_t prefill_embed_launch(const PrefillTok* toks, int T, const float* embed, int text_vocab,
                                 const float* lang, int n_lang, const int* lang_ids,
                                 const int64_t* frames, int Q, const float* table, int V,
                                 float scale, const float* slot, const float* bos_add, float* X,
                                 int D, int* err, cudaStream_t s);
cudaError_t speaker_launch(const float* v, int SD, const float* W, int D, const float* slot,
                           float* out, cudaStream_t s);
cudaError_t sgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl = false);
// The batched / prefill GEMM (GemmArgs::variant picks the kernel; 0 =
// by rows): the FP32 FFMA kernel of fgemm.cu for T <= 16, else the 3xTF32
// tcgen05 GEMM of tgemm.cu; K a multiple of 32 (256 for the FFMA kernel).
cudaError_t tgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl = false);
bool fgemm_supported(const GemmArgs& a);
cudaError_t fgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl = false);
cudaError_t prefill_qk_launch(const float* qkv, int ld, const PrefillTok* toks, int T,
                              const float* qn, const float* kn, float eps, const float* rc,
                              const float* rs, int H, const KVLayout& kv, int layer, float* Qo,
                              cudaStream_t s);
cudaError_t prefill_attn_launch(const float* Q, const int* row_off, const int* row_len,
                                const int* row_id, int n_rows, int max_L, int H, int n_rep,
                                const KVLayout& kv, int layer, float scale, float* out,
                                cudaStream_t s);
cudaError_t trunk_init_attrs();

cudaError_t gather_rows_launch(const float* X, const int* src, const int* dst, int n, float* out,
                               int D, cudaStream_t s);

}  // namespace skb
