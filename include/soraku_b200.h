/*
 * soraku_b200.h -- C ABI of the B200 (sm_100a) backend for soraku-TTS's
 * per-frame autoregressive token loop.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t and
 * returns an int status (SKB_OK on success).  Nothing here allocates the
 * caller's outputs; the engine allocates and owns its own state (KV pages,
 * scratch, the captured CUDA graph).  Tensors are FP32, row-major and
 * contiguous; code tensors are int64 as in the reference.
 *
 * Reference interfaces replaced (paths inside the soraku-TTS checkout):
 *   soraku_inference/acceleration/tilelang_kernels.py  -- the 8 op factories
 *   soraku_inference/acceleration/graph_frame.py       -- GraphFrameEngine
 *   soraku_inference/model.py:579-595,686-708          -- CFG + _sample_logits
 */
#ifndef SORAKU_B200_H
#define SORAKU_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef __CUDA_RUNTIME_H__
typedef struct CUstream_st *cudaStream_t;
#endif

/* Status codes.  The Python shim maps SKB_ERR_ARG to ValueError and the rest
 * to RuntimeError, as the reference raises (graph_frame.py:155-156,301-302). */
#define SKB_OK 0
#define SKB_ERR_ARG 1      /* bad shape, size or pointer alignment          */
#define SKB_ERR_STATE 2    /* call order, e.g. step before capture          */
#define SKB_ERR_CUDA 3     /* a CUDA runtime call failed                    */
#define SKB_ERR_CAPACITY 4 /* KV cache / frame buffer full                  */
#define SKB_ERR_NOMEM 5    /* device allocation failed                      */

/* Message for the last non-OK status returned on this host thread. */
const char *skb_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int skb_abi_version(void);

/* ------------------------------------------------------------------------
 * Op surface.  Same names, argument order and meaning as the TileLang
 * factories; the factory's static shape parameters become size arguments.
 * GEMV inner sizes (D of swiglu/classifier, I of down) must be multiples of
 * 4 and <= 3072; pointers 16-byte aligned (SKB_ERR_ARG otherwise).
 * ---------------------------------------------------------------------- */

/* tilelang_kernels.py:34-55  add_rmsnorm(B,D,eps)(hidden,prefix,weight)
 * out = rmsnorm(hidden + prefix) * weight */
int skb_add_rmsnorm(const float *hidden, const float *prefix, const float *weight, float *out,
                    int B, int D, float eps, cudaStream_t stream);

/* tilelang_kernels.py:58-78  rmsnorm(B,D,eps)(x,weight)
 * out = rmsnorm(x) * weight */
int skb_rmsnorm(const float *x, const float *weight, float *out, int B, int D, float eps,
                cudaStream_t stream);

/* tilelang_kernels.py:81-112  swiglu_gemv(B,I,D)(x,wg,wu)
 * out[b] = silu(x[b] @ wg^T) * (x[b] @ wu^T);  wg, wu: [I, D] */
int skb_swiglu_gemv(const float *x, const float *wg, const float *wu, float *out, int B, int I,
                    int D, cudaStream_t stream);

/* tilelang_kernels.py:115-143  down_residual_gemv(B,D,I)(act,wd,residual)
 * out[b] = act[b] @ wd^T + residual[b];  wd: [D, I] */
int skb_down_residual_gemv(const float *act, const float *wd, const float *residual, float *out,
                           int B, int D, int I, cudaStream_t stream);

/* tilelang_kernels.py:146-173  classifier_gemv(B,V,D)(body,wq,bias)
 * out[b] = body[b] @ wq^T + bias;  wq: [V, D] */
int skb_classifier_gemv(const float *body, const float *wq, const float *bias, float *out, int B,
                        int V, int D, cudaStream_t stream);

/* tilelang_kernels.py:176-196  frame_embed(R,Q,V,D,scale)(codes,table)
 * out[r] = scale * sum_q table[q, codes[r, q], :]  (sum in q order, then scale) */
int skb_frame_embed(const int64_t *codes, const float *table, float *out, int R, int Q, int V,
                    int D, float scale, cudaStream_t stream);

/* tilelang_kernels.py:199-216  prefix_add(B,V,D,scale)(prefix,table_q,codes)
 * out[b] = prefix[b] + table_q[codes[0]] * scale */
int skb_prefix_add(const float *prefix, const float *table_q, const int64_t *code, float *out,
                   int B, int V, int D, float scale, cudaStream_t stream);

/* tilelang_kernels.py:219-254  sampling_prep(V,bos,pad,eos)(logits,temperature,mask_eos)
 * out = logits / temperature[0]; BOS, PAD (and EOS when mask_eos[0] > 0) -> -1e30 */
int skb_sampling_prep(const float *logits, const float *temperature, const int32_t *mask_eos,
                      float *out, int V, int bos_id, int pad_id, int eos_id, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Fused CFG + mask + temperature + top-k + top-p + draw, one CTA per request.
 * Replaces model.py:579-595 with _sample_logits (model.py:686-708) and the
 * graph engine's in-graph sampling (graph_frame.py:214-241).  The draw uses a
 * Philox4x32-10 uniform with counter (q, frame, request, 0) and key = seed.
 * ---------------------------------------------------------------------- */
typedef struct {
    float cfg_scale;   /* merged = u + s (c - u); ignored with 1 row/request */
    float temperature; /* <= 0 selects argmax                               */
    int top_k;         /* active iff 0 < top_k < V                           */
    float top_p;       /* active iff 0 < top_p < 1                           */
    int mask_eos;      /* nonzero: EOS -> -inf                               */
    uint32_t request;  /* Philox counter word 2                              */
    uint32_t frame;    /* Philox counter word 1                              */
    uint32_t q;        /* Philox counter word 0                              */
    uint64_t seed;     /* Philox key                                         */
} skb_sample_params;

/* logits: device [n_req * rows_per_req, V] (cond row first, then uncond);
 * params: device [n_req]; codes_out: device int64 [n_req];
 * uniform_out: optional device float [n_req] (the uniform each draw used). */
int skb_cfg_sample(const float *logits, int rows_per_req, int n_req, int V,
                   const skb_sample_params *params, int bos_id, int pad_id, int eos_id,
                   int64_t *codes_out, float *uniform_out, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * One decode-attention step of a Qwen3 layer (the attention half of
 * modeling_qwen3.py Qwen3Attention.forward :240-291 for one new token per
 * row): q/k RMSNorm over each head, neox RoPE at pos[row], append k/v at
 * pos[row] of the paged cache, GQA softmax(q k^T / sqrt(hd)) v over positions
 * 0..pos[row].  The engine runs the same kernel for every layer.
 *   qkv        device [rows, (n_heads + 2 n_kv_heads) * head_dim]  (q | k | v)
 *   rope_cos/sin device [max_len, head_dim / 2]  cos/sin of inv_freq[i] * p
 *   pos        device int32 [rows]  position of the new token (< max_len)
 *   kv_pool    device [n_pages][2][n_kv_heads][page_size][head_dim]
 *   page_table device int32 [rows, max_pages]
 *   part       scratch [rows * n_kv_heads * splits * (n_heads/n_kv_heads) * (head_dim + 2)]
 *   tickets    scratch int32 [rows * n_kv_heads], zero before the call (left zero)
 *   out        device [rows, n_heads * head_dim]
 * head_dim must be 128 and n_heads / n_kv_heads 1 or 2; qkv, the norm weights,
 * the RoPE tables and kv_pool 16-byte aligned. */
int skb_decode_attention(const float *qkv, int rows, int n_heads, int n_kv_heads, int head_dim,
                         const float *q_norm, const float *k_norm, float eps, const float *rope_cos,
                         const float *rope_sin, int max_len, const int32_t *pos, float *kv_pool,
                         const int32_t *page_table, int max_pages, int page_size, int n_pages,
                         int splits, float *part, int32_t *tickets, float *out, cudaStream_t stream);

/* Decode attention for callers that must not allocate device memory.  It has
 * no counterpart in the reference.  Some hosts cannot call cudaMalloc when a
 * frame is decoded: an audio or streaming thread cannot afford the device-wide
 * synchronisation an allocation may cause, and an application that reserves
 * all device memory up front through its own allocator forbids raw
 * allocations.  Such callers pass the same inputs and outputs as to
 * skb_decode_attention but no scratch: the split partials and tickets live in
 * one library-owned device array of SKB_NOALLOC_SCRATCH_BYTES (2 MiB + 1 KiB),
 * which every GPU that loads this library holds until the process exits.
 * Limit: rows * n_kv_heads * splits * (n_heads / n_kv_heads) * (head_dim + 2)
 * floats must fit in 2 MiB and rows * n_kv_heads tickets in 1 KiB; larger
 * calls return SKB_ERR_ARG.  The first call on a device looks up the array's
 * device address (a one-time set-up), so make that first call before any
 * stream capture.  All calls share the array and it keeps the last call's
 * contents: calls that overlap on the GPU (different streams, or different
 * host threads on one device) race and must be serialised by the caller.
 * Every argument is checked before the array is touched.  The looked-up
 * address is cached per device and goes stale after cudaDeviceReset on that
 * device: do not call this entry point on a device after resetting it.
 * No cudaMalloc, cudaFree or allocating library routine is called. */
#define SKB_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u + 1024u)
int skb_decode_attention_noalloc(const float *qkv, int rows, int n_heads, int n_kv_heads,
                                 int head_dim, const float *q_norm, const float *k_norm, float eps,
                                 const float *rope_cos, const float *rope_sin, int max_len,
                                 const int32_t *pos, float *kv_pool, const int32_t *page_table,
                                 int max_pages, int page_size, int n_pages, int splits, float *out,
                                 cudaStream_t stream);

/* Test hooks: the device exp used by the sampler, and raw Philox4x32-10.
 * ctr_key: device uint32 [n, 6] = (c0, c1, c2, c3, k0, k1); out: [n, 4]. */
int skb_test_exp(const float *x, float *y, int n, cudaStream_t stream);
/* out[M, N] = x[M, K] @ w[N, K]^T on the batched/prefill GEMM: tensor_cores
 * 1 = the kernel chosen by M (the FP32 FFMA few-row kernel for M <= 16 and
 * K % 256 == 0, else the 3xTF32 tcgen05 kernel), 2 = the tcgen05 kernel,
 * 3 = the FFMA few-row kernel (M <= 32, K % 256 == 0); splits: K splits per
 * tcgen05 output tile, 0 = chosen by occupancy; 0 = the SIMT FP32 prefill
 * kernel.  K % 32 == 0. */
int skb_test_gemm(const float *x, const float *w, float *out, int M, int N, int K, int tensor_cores, int splits,
                  cudaStream_t stream);
int skb_test_philox(const uint32_t *ctr_key, uint32_t *out, int n, cudaStream_t stream);
/* Failure-path hook: a one-thread kernel waits limit_us (1..10^6) on an
 * mbarrier phase nothing completes, through the decode kernels' bounded wait,
 * which gives up and sets *err (device int); the call synchronises `stream`
 * and returns SKB_ERR_CUDA when the flag is set, SKB_OK otherwise. */
int skb_test_wait_timeout(int *err, int limit_us, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Decode engine: replaces GraphFrameEngine (graph_frame.py:23-328).
 * ---------------------------------------------------------------------- */
typedef struct skb_engine skb_engine;

/* Per-layer weight pointers, in this order, borrowed (never copied):
 * q_proj [Hq*hd, d], k_proj [Hkv*hd, d], v_proj [Hkv*hd, d], o_proj [d, Hq*hd],
 * q_norm [hd], k_norm [hd], gate [F, d], up [F, d], down [d, F],
 * input_layernorm [d], post_attention_layernorm [d]. */
#define SKB_LAYER_PTRS 11

typedef struct {
    int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn_dim;
    int text_vocab, n_codebooks, audio_vocab, depth_inner, speaker_dim;
    float rms_eps;     /* trunk RMSNorm eps (1e-6)                         */
    float depth_eps;   /* depth-head RMSNorm eps (FLT_EPSILON)             */
    float frame_scale; /* n_codebooks ** -0.5                              */
    int bos_id, eos_id, pad_id;
    int n_lang;        /* 0 or 4 language token ids                        */
    int lang_ids[4];
    const float *embed_tokens;    /* [text_vocab, d]                       */
    const float *lang_embed;      /* [4, d] or NULL                        */
    const float *final_norm;      /* [d]                                   */
    const float *table;           /* [Q, audio_vocab, d]                   */
    const float *depth_bias;      /* [Q, audio_vocab]                      */
    const float *depth_norm_in;   /* [d]                                   */
    const float *depth_norm_out;  /* [d]                                   */
    const float *depth_gate;      /* [depth_inner, d]                      */
    const float *depth_up;        /* [depth_inner, d]                      */
    const float *depth_down;      /* [d, depth_inner]                      */
    const float *speaker_proj;    /* [d, speaker_dim] or NULL              */
    const float *speaker_slot;    /* [d] or NULL (slot mode)               */
    int speaker_slot_mode;        /* 1: slot between text and audio; 0: add to BOS frame */
    const float *rope_inv_freq;   /* host pointer, [head_dim / 2]          */
    const float *const *layers;   /* host array [n_layers * SKB_LAYER_PTRS] */
} skb_model_desc;

typedef struct {
    int max_requests;     /* requests decoded together                     */
    int rows_per_request; /* 2 with CFG (cond, uncond), 1 without          */
    int max_len;          /* KV capacity per row, in positions             */
    int max_frames;       /* code history capacity per request             */
    int max_prefill;      /* prompt positions per row                      */
    int page_size;        /* KV page size in positions (power of two)      */
    int attn_splits;      /* 0 = choose; KV splits per (row, kv head)      */
    int use_pdl;          /* programmatic dependent launch between kernels */
    int l2_prefetch;      /* bulk-prefetch the next kernel's weights       */
    int gemm_min_rows;    /* batches of at least this many rows run the
                             tensor-core GEMM path (0 = 5); 1 makes every
                             batch take it, so a row's arithmetic does not
                             depend on the batch width                      */
    int prefill_batch;    /* requests one skb_engine_prefill_many pass can
                             hold (0 = 1); sizes the prefill scratch        */
    int kv_pages;         /* 0: every row owns ceil(max_len / page_size)
                             pages; > 0: a shared pool of this many pages
                             per layer, mapped to rows by
                             skb_engine_map_pages (unmapped positions are
                             refused by prefill and step)                   */
    int split_depth_head; /* 0: a batch of one CFG request on the GEMV path
                             runs the frame's 16 depth steps as one
                             persistent cooperative launch (gate/up slices
                             resident in shared memory, grid barriers
                             between phases); 1: 64 separate kernels    */
} skb_engine_opts;

int skb_engine_create(const skb_model_desc *model, const skb_engine_opts *opts, skb_engine **out);
int skb_engine_destroy(skb_engine *eng);

/* graph_frame.py:118-198 prefill, per request.  Host int64 arrays:
 * cond_ids [n_cond], uncond_ids [n_uncond] (ignored with 1 row/request),
 * prompt_codes [n_prompt, Q] (may be NULL with n_prompt 0), speaker: host
 * float [speaker_dim] or NULL.  Embeds as model.py:623-653 (language-ID
 * substitution of embed_text included), runs the trunk over every position,
 * fills the KV pages and leaves the request ready for frame 0. */
int skb_engine_prefill(skb_engine *eng, int request, const int64_t *cond_ids, int n_cond,
                       const int64_t *uncond_ids, int n_uncond, const int64_t *prompt_codes,
                       int n_prompt, const float *speaker, cudaStream_t stream);

/* The prompts of n <= opts.prefill_batch distinct requests in one pass over
 * the trunk (their tokens concatenated, so every GEMM sees all of them);
 * arrays of n host pointers / counts as for skb_engine_prefill, without
 * speaker vectors (route-D requests go through skb_engine_prefill). */
int skb_engine_prefill_many(skb_engine *eng, int n, const int *requests, const int64_t *const *cond_ids,
                            const int *n_cond, const int64_t *const *uncond_ids, const int *n_uncond,
                            const int64_t *const *prompt_codes, const int *n_prompt, cudaStream_t stream);

/* graph_frame.py:307-328 set_temperature/set_sampling/set_seed, per request.
 * top_k <= 0 or top_p outside (0,1) disable the filter; *_q0 apply to q0.
 * eos_rule 0: q0 may emit EOS only when the host flag of skb_engine_step is 0;
 * eos_rule 1: only when the request's frame index >= min_new_frames. */
int skb_engine_set_sampling(skb_engine *eng, int request, float cfg_scale, float temperature,
                            float temperature_q0, int top_k, float top_p, int top_k_q0,
                            float top_p_q0, uint64_t seed, int min_new_frames, int eos_rule);

/* graph_frame.py:274-296 capture: records frames_per_graph whole frames
 * (16 depth steps with sampling, frame embedding, one trunk step) for the
 * first n_active requests as one CUDA graph.  The engine keeps the 16 most
 * recently used (n_active, frames_per_graph) graphs, so returning to a batch
 * width captured before costs no new capture. */
int skb_engine_capture(skb_engine *eng, int n_active, int frames_per_graph, cudaStream_t stream);

/* graph_frame.py:298-305 step_frame: replays the graph once (frames_per_graph
 * frames).  mask_eos_q0 is the host EOS flag of eos_rule 0.  Device error
 * flags (view 6: a position out of range, a prefill input out of range, a
 * weight copy that did not arrive within its bounded wait) surface here as
 * SKB_ERR_CUDA: each step queues a copy of the flags behind its replay, and
 * a later step reports a raised flag once that copy has landed (without
 * waiting for it); after that every step fails, as graph_frame.py:155-156,
 * 301-302 raise RuntimeError for an unusable engine. */
int skb_engine_step(skb_engine *eng, int mask_eos_q0, cudaStream_t stream);

/* Runs the same frame body eagerly (kernel by kernel, no graph). */
int skb_engine_step_eager(skb_engine *eng, int n_active, int mask_eos_q0, cudaStream_t stream);

/* Copies codes [n_frames, Q] of a request, frames [first, first+n), to a
 * device or host int64 buffer (cudaMemcpyAsync on stream). */
int skb_engine_read_codes(skb_engine *eng, int request, int first_frame, int n_frames,
                          int64_t *dst, cudaStream_t stream);

/* Frames decoded so far for a request (host-side counter). */
int skb_engine_frames(skb_engine *eng, int request);

/* Continuous batching (requests joining and leaving a running batch).
 * set_rng_stream: the request's Philox stream word (counter = (stream, frame,
 * q) under its seed; default: the slot index), so a request's draws need not
 * depend on the slot it occupies.
 * status: device frame counters and EOS flags of requests [0, n) into host
 * arrays (synchronises the stream); returns SKB_ERR_CUDA if a device error
 * flag is raised.
 * move_request: moves request `src`'s decode state (sampling state, codes,
 * prefix, residual stream, positions, KV pages by page-table exchange) into
 * slot `dst`, leaving `src` free; for compacting the active slots. */
int skb_engine_set_rng_stream(skb_engine *eng, int request, uint32_t stream);
int skb_engine_status(skb_engine *eng, int n, int32_t *frames, int32_t *done, cudaStream_t stream);
int skb_engine_move_request(skb_engine *eng, int dst, int src, cudaStream_t stream);
/* Shared KV pool (opts.kv_pages > 0): row `row`'s logical pages [first,
 * first + n) become pool pages pages[0..n) (host int32; -1 unmaps).  A
 * page must not be mapped to two rows at once; the caller owns the free
 * list (soraku_tts_b200/scheduler.py PagePool). */
int skb_engine_map_pages(skb_engine *eng, int row, int first, int n, const int32_t *pages);

/* Device views of engine state for tests: which = 0 x (residual stream)
 * [R, d]; 1 hidden [R, d]; 2 logits [R, V] of the last depth step; 3 pos
 * int32 [R]; 4 logits history [Q, R, V] of the last frame (debug capture must
 * be on); 5 prefix [n_req, d]; 6 error flags int32 [8]; 7 request state;
 * 8 kernel timeline uint64 [kernels per frame][16] of the last replayed
 * frame with debug on: earliest CTA start, earliest and latest release from
 * the dependent-launch wait, latest CTA end, then the latest CTA to reach
 * kernel-specific points (%globaltimer ns; the caller resets it to
 * {max, max, 0, ...} before the frame); 9 persistent depth-head timeline
 * uint64 [4 Q][2] of the last frame with debug on (CTA 0's release of each
 * phase -- UP, DN, CLS, SAMPLE per codebook -- and the end of its work,
 * %globaltimer ns). */
int skb_engine_view(skb_engine *eng, int which, void **ptr, int64_t *numel);

/* Keep the per-(q) logits of the last frame in the history buffer (view 4). */
int skb_engine_set_debug(skb_engine *eng, int on);

/* Number of kernels one frame launches. */
int skb_engine_kernels_per_frame(skb_engine *eng);

/* Kernel launches one skb_engine_step makes with the captured graph
 * (frames_per_graph x kernels per frame; 0 before capture). */
int skb_engine_launches_per_step(skb_engine *eng);

#ifdef __cplusplus
}
#endif
#endif /* SORAKU_B200_H */
