// Trunk kernels: decode attention for more than 8 splits per (row, kv head)
// (split over the KV positions, last-CTA combine), the prefill path
// (embedding, q/k norm + RoPE + KV write, causal attention; its projections
// run on the tensor-core GEMM of tgemm.cu), and the SIMT FP32 GEMM that
// skb_test_gemm keeps as the comparison path of the tensor-core one.
#include "ops.cuh"
#include "trunk.cuh"
#include "trunk_api.cuh"

namespace skb {

// grid (S, KVH, R), 256 threads: one work item per CTA.
__global__ void __launch_bounds__(256) decode_attn_kernel(const DecodeAttnArgs a) {
    __shared__ AttnSmem sm;
    const int s = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int nblk = gridDim.x * gridDim.y * gridDim.z;
    if (threadIdx.x == 0) stamp_min(a.ts);
    prefetch_share(a.pf, (r * gridDim.y + g) * gridDim.x + s, nblk);
    pdl_wait();
    if (threadIdx.x == 0) stamp_wait(a.ts);
    pdl_trigger();
    decode_attn_item<BlockSync>(a, s, g, r, sm);
    if (a.ts) {
        __syncthreads();
        if (threadIdx.x == 0) stamp_max(a.ts + 3);
    }
}

cudaError_t decode_attn_launch(const DecodeAttnArgs& a, int R, cudaStream_t s, bool pdl) {
    return launch(decode_attn_kernel, dim3(a.S, a.kv.KVH, R), dim3(256), 0, s, pdl, a);
}

// ------------------------------------------------------------------ prefill
// Token embeddings (model.py:623-653): text ids through the text table with
// language-id substitution (embed_text, model.py:326-338); audio frames as
// scale * sum_q table[q, code]; the speaker slot vector.
__global__ void __launch_bounds__(256) prefill_embed_kernel(
    const PrefillTok* __restrict__ toks, const float* __restrict__ embed, int text_vocab,
    const float* __restrict__ lang, int n_lang, int4 lang_ids, const int64_t* __restrict__ frames,
    int Q, const float* __restrict__ table, int V, float scale, const float* __restrict__ slot,
    const float* __restrict__ bos_add, float* __restrict__ X, int D, int* err) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const PrefillTok tk = toks[t];
    float* xo = X + (size_t)t * D;
    if (tk.kind == 0) {
        int id = tk.val;
        int li = -1;
        if (n_lang == 4) {
            if (id == lang_ids.x) li = 0;
            else if (id == lang_ids.y) li = 1;
            else if (id == lang_ids.z) li = 2;
            else if (id == lang_ids.w) li = 3;
        }
        if (li < 0 && (id < 0 || id >= text_vocab)) {
            if (threadIdx.x == 0) atomicExch(err, 2);
            id = 0;
        }
        const float* src = li >= 0 ? lang + (size_t)li * D : embed + (size_t)id * D;
        for (int i = threadIdx.x; i < D; i += 256) xo[i] = src[i];
    } else if (tk.kind == 1) {
        const int64_t* fc = frames + (size_t)tk.val * Q;
        for (int i = threadIdx.x; i < D; i += 256) {
            float acc = 0.f;
            for (int q = 0; q < Q; ++q) {
                long long c = fc[q];
                if (c < 0 || c >= V) {
                    atomicExch(err, 3);
                    c = 0;
                }
                const float v = table[((size_t)q * V + (size_t)c) * D + i];
                acc = (q == 0) ? v : acc + v;
            }
            acc = acc * scale;
            if (bos_add != nullptr && tk.val == 0) acc = acc + bos_add[i];
            xo[i] = acc;
        }
    } else {
        for (int i = threadIdx.x; i < D; i += 256) xo[i] = slot[i];
    }
}

// Speaker projection (model.py:404-421): out = W @ normalize(v) (+ slot), 1 CTA.
__global__ void __launch_bounds__(256) speaker_kernel(const float* __restrict__ v, int SD,
                                                      const float* __restrict__ W, int D,
                                                      const float* __restrict__ slot_emb,
                                                      float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float vs[1024];
    __shared__ float red[8];
    float ss = 0.f;
    for (int i = threadIdx.x; i < SD; i += 256) {
        const float x = v[i];
        vs[i] = x;
        ss += x * x;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float nrm = fmaxf(sqrtf(tot), 1e-12f);
    for (int i = threadIdx.x; i < SD; i += 256) vs[i] = vs[i] / nrm;
    __syncthreads();
    for (int o = threadIdx.x; o < D; o += 256) {
        const float* wr = W + (size_t)o * SD;
        float acc = 0.f;
        for (int i = 0; i < SD; ++i) acc = fmaf(wr[i], vs[i], acc);
        out[o] = slot_emb ? acc + slot_emb[o] : acc;
    }
}

// SIMT FP32 GEMM (skb_test_gemm tensor_cores = 0):
// C[t][n] = sum_k A[t][k] W(n)[k], 64x64 tiles, BK 16, 4x4 per thread.
__device__ __forceinline__ const float* gemm_row(const GemmArgs& a, int n) {
    if (a.interleave) return ((n & 1) ? a.w1 : a.w0) + (size_t)(n >> 1) * a.K;
    if (n < a.seg1) return a.w0 + (size_t)n * a.K;
    if (n < a.seg2) return a.w1 + (size_t)(n - a.seg1) * a.K;
    return a.w2 + (size_t)(n - a.seg2) * a.K;
}

__global__ void __launch_bounds__(256) sgemm_kernel(const GemmArgs a) {
    __shared__ __align__(16) float As[16][64 + 4];
    __shared__ __align__(16) float Ws[16][64 + 4];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int n0 = blockIdx.x * 64, t0 = blockIdx.y * 64;
    const int lr = tid >> 2, lk = (tid & 3) * 4;  // loader: row lr, k offset lk
    const int tA = t0 + lr, nW = n0 + lr;
    const float* arow = (tA < a.T) ? a.A + (size_t)tA * a.lda : nullptr;
    const float* wrow = (nW < a.N) ? gemm_row(a, nW) : nullptr;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int k0 = 0; k0 < a.K; k0 += 16) {
        const float4 av = arow ? *reinterpret_cast<const float4*>(arow + k0 + lk) : make_float4(0, 0, 0, 0);
        const float4 wv = wrow ? __ldg(reinterpret_cast<const float4*>(wrow + k0 + lk)) : make_float4(0, 0, 0, 0);
        As[lk + 0][lr] = av.x;
        As[lk + 1][lr] = av.y;
        As[lk + 2][lr] = av.z;
        As[lk + 3][lr] = av.w;
        Ws[lk + 0][lr] = wv.x;
        Ws[lk + 1][lr] = wv.y;
        Ws[lk + 2][lr] = wv.z;
        Ws[lk + 3][lr] = wv.w;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float4 x = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&Ws[k][tx * 4]);
            const float xa[4] = {x.x, x.y, x.z, x.w};
            const float wa[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= a.T) continue;
        if (a.mode == 3) {
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
                const int n = n0 + tx * 4 + j;
                if (n + 1 < a.N) a.out[(size_t)t * a.ldo + (n >> 1)] = silu(acc[i][j]) * acc[i][j + 1];
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + tx * 4 + j;
                if (n >= a.N) continue;
                float v = acc[i][j];
                if (a.mode == 1) v += a.resid[(size_t)t * a.ldr + n];
                if (a.mode == 2) v += __ldg(a.bias + n);
                a.out[(size_t)t * a.ldo + n] = v;
            }
        }
    }
}

cudaError_t sgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl) {
    if (a.K % 16 != 0) return cudaErrorInvalidValue;
    return launch(sgemm_kernel, dim3((a.N + 63) / 64, (a.T + 63) / 64), dim3(256), 0, s, pdl, a);
}

// Per token: q/k RMSNorm + RoPE at the token's position; q -> Qo, k/v -> KV.
// grid T, 256 threads (warp w handles head vectors w, w+8, ...).
__global__ void __launch_bounds__(256) prefill_qk_kernel(const float* __restrict__ qkv, int ld,
                                                         const PrefillTok* __restrict__ toks,
                                                         const float* qn, const float* kn, float eps,
                                                         const float* rope_cos, const float* rope_sin,
                                                         int H, KVLayout kv, int layer,
                                                         float* __restrict__ Qo) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const PrefillTok tk = toks[t];
    const float* row = qkv + (size_t)t * ld;
    const float* cosr = rope_cos + (size_t)tk.pos * 64;
    const float* sinr = rope_sin + (size_t)tk.pos * 64;
    const int nvec = H + 2 * kv.KVH;
    for (int v = warp; v < nvec; v += 8) {
        float4 x = reinterpret_cast<const float4*>(row + v * 128)[lane];
        if (v < H) {
            x = norm_rope_head(x, qn, eps, cosr, sinr, lane, true, true);
            reinterpret_cast<float4*>(Qo + (size_t)t * H * 128 + v * 128)[lane] = x;
        } else if (v < H + kv.KVH) {
            x = norm_rope_head(x, kn, eps, cosr, sinr, lane, true, true);
            reinterpret_cast<float4*>(kv.at(layer, tk.row, tk.pos, 0, v - H))[lane] = x;
        } else {
            reinterpret_cast<float4*>(kv.at(layer, tk.row, tk.pos, 1, v - H - kv.KVH))[lane] = x;
        }
    }
}

// Causal attention of a row's prompt: grid (ceil(L/8), KVH, n_rows); each
// CTA serves 8 query positions x n_rep heads (<= 16 query vectors, 2 per
// warp, staged pre-scaled in shared memory); keys and values stream through
// shared memory 32 positions at a time with an online softmax, the next
// block's loads in flight during this block's math.  The CTA of the last
// query block walks every key block, so the query block is kept small: that
// CTA's serial chain sets the kernel's time.
constexpr int PATTN_QP = 8;                 // query positions per CTA
constexpr int PATTN_QVEC = 2 * PATTN_QP;    // query vectors per CTA (n_rep <= 2)
constexpr int PATTN_SMEM = (PATTN_QVEC * 128 + 32 * 129 + 32 * 128) * 4;

__global__ void __launch_bounds__(256) prefill_attn_kernel(const float* __restrict__ Q,
                                                           const int* __restrict__ row_off,
                                                           const int* __restrict__ row_len,
                                                           const int* __restrict__ row_id,
                                                           int H, int n_rep, KVLayout kv, int layer,
                                                           float scale, float* __restrict__ out) {
    extern __shared__ float psm[];
    float* Qs = psm;                     // [PATTN_QVEC][128]
    float* Ks = psm + PATTN_QVEC * 128;  // [32][129]
    float* Vs = Ks + 32 * 129;        // [32][128]
    pdl_wait();
    pdl_trigger();
    const int qb = blockIdx.x, g = blockIdx.y, ri = blockIdx.z;
    const int L = row_len[ri], off = row_off[ri], row = row_id[ri];
    const int q0 = qb * PATTN_QP;
    if (q0 >= L) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int QV = PATTN_QVEC / 8;
    // query vector v: position q0 + v / n_rep, head g * n_rep + v % n_rep
    for (int i = threadIdx.x; i < PATTN_QVEC * 128; i += 256) {
        const int v = i >> 7, d = i & 127;
        const int p = q0 + v / n_rep, h = g * n_rep + v % n_rep;
        Qs[i] = (p < L && v < PATTN_QP * n_rep) ? Q[(size_t)(off + p) * H * 128 + h * 128 + d] * scale : 0.f;
    }
    float m[QV], l[QV], o[QV][4];
    int qpos[QV];
#pragma unroll
    for (int j = 0; j < QV; ++j) {
        const int v = warp * QV + j;
        qpos[j] = (v < PATTN_QP * n_rep) ? q0 + v / n_rep : 0x7fffffff;
        m[j] = -INFINITY;
        l[j] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.f;
    }
    const int last_q = min(L - 1, q0 + PATTN_QP - 1);
    // K/V blocks of 32 positions: thread t loads position t / 8 of the block,
    // float4 columns t % 8 + 8 j (one page lookup per thread), into registers
    // one block ahead, so the next block's loads are in flight during this
    // block's math.
    const int lk = threadIdx.x >> 3, lc = threadIdx.x & 7;
    float4 kr[4], vr[4];
    auto load_block = [&](int k0) {
        const int p = k0 + lk;
        const bool ok = p < L;
        const float4* kb = ok ? reinterpret_cast<const float4*>(kv.at(layer, row, p, 0, g)) : nullptr;
        const float4* vb = ok ? reinterpret_cast<const float4*>(kv.at(layer, row, p, 1, g)) : nullptr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kr[j] = ok ? __ldcg(kb + lc + 8 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
            vr[j] = ok ? __ldcg(vb + lc + 8 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    load_block(0);
    for (int k0 = 0; k0 <= last_q; k0 += 32) {
        __syncthreads();  // the previous block's math is done with Ks / Vs
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = 4 * (lc + 8 * j);
            float* kd = Ks + lk * 129 + d;
            kd[0] = kr[j].x;
            kd[1] = kr[j].y;
            kd[2] = kr[j].z;
            kd[3] = kr[j].w;
            *reinterpret_cast<float4*>(Vs + lk * 128 + d) = vr[j];
        }
        __syncthreads();
        if (k0 + 32 <= last_q) load_block(k0 + 32);
        const int p = k0 + lane;
        float sdot[QV];
#pragma unroll
        for (int j = 0; j < QV; ++j) sdot[j] = 0.f;
        const float* qw = Qs + (warp * QV) * 128;
#pragma unroll 4
        for (int d = 0; d < 128; ++d) {
            const float kd = Ks[lane * 129 + d];
#pragma unroll
            for (int j = 0; j < QV; ++j) sdot[j] = fmaf(qw[j * 128 + d], kd, sdot[j]);
        }
#pragma unroll
        for (int j = 0; j < QV; ++j) {
            const bool valid = p <= qpos[j] && p < L && qpos[j] < L;
            const float sv = valid ? sdot[j] : -INFINITY;
            const float mt = warp_max(sv);
            const float mn = fmaxf(m[j], mt);
            if (mn == -INFINITY) continue;
            const float pe = valid ? expf(sv - mn) : 0.f;
            const float corr = expf(m[j] - mn);
            l[j] = l[j] * corr + warp_sum(pe);
            m[j] = mn;
#pragma unroll
            for (int c = 0; c < 4; ++c) o[j][c] *= corr;
            for (int kk = 0; kk < 32; ++kk) {
                const float pk = __shfl_sync(FULL, pe, kk);
#pragma unroll
                for (int c = 0; c < 4; ++c) o[j][c] = fmaf(pk, Vs[kk * 128 + lane + 32 * c], o[j][c]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < QV; ++j) {
        if (qpos[j] >= L) continue;
        const int v = warp * QV + j;
        const int h = g * n_rep + v % n_rep;
        const float inv = 1.0f / l[j];
#pragma unroll
        for (int c = 0; c < 4; ++c)
            out[(size_t)(off + qpos[j]) * H * 128 + h * 128 + lane + 32 * c] = o[j][c] * inv;
    }
}

// x_trunk[row] = X[last token of row]
__global__ void gather_rows_kernel(const float* __restrict__ X, const int* __restrict__ src,
                                   const int* __restrict__ dst, float* __restrict__ out, int D) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        out[(size_t)dst[r] * D + i] = X[(size_t)src[r] * D + i];
}

cudaError_t prefill_embed_launch(const PrefillTok* toks, int T, const float* embed, int text_vocab,
                                 const float* lang, int n_lang, const int* lang_ids,
                                 const int64_t* frames, int Q, const float* table, int V,
                                 float scale, const float* slot, const float* bos_add, float* X,
                                 int D, int* err, cudaStream_t s) {
    const int4 li = make_int4(lang_ids[0], lang_ids[1], lang_ids[2], lang_ids[3]);
    return launch(prefill_embed_kernel, dim3(T), dim3(256), 0, s, false, toks, embed, text_vocab,
                  lang, n_lang, li, frames, Q, table, V, scale, slot, bos_add, X, D, err);
}

cudaError_t speaker_launch(const float* v, int SD, const float* W, int D, const float* slot,
                           float* out, cudaStream_t s) {
    if (SD > 1024) return cudaErrorInvalidValue;
    return launch(speaker_kernel, dim3(1), dim3(256), 0, s, false, v, SD, W, D, slot, out);
}

cudaError_t prefill_qk_launch(const float* qkv, int ld, const PrefillTok* toks, int T,
                              const float* qn, const float* kn, float eps, const float* rc,
                              const float* rs, int H, const KVLayout& kv, int layer, float* Qo,
                              cudaStream_t s) {
    return launch(prefill_qk_kernel, dim3(T), dim3(256), 0, s, false, qkv, ld, toks, qn, kn, eps, rc,
                  rs, H, kv, layer, Qo);
}

cudaError_t prefill_attn_launch(const float* Q, const int* row_off, const int* row_len,
                                const int* row_id, int n_rows, int max_L, int H, int n_rep,
                                const KVLayout& kv, int layer, float scale, float* out,
                                cudaStream_t s) {
    if (n_rep < 1 || PATTN_QP * n_rep > PATTN_QVEC) return cudaErrorInvalidValue;
    return launch(prefill_attn_kernel, dim3((max_L + PATTN_QP - 1) / PATTN_QP, kv.KVH, n_rows), dim3(256),
                  PATTN_SMEM, s,
                  false, Q, row_off, row_len, row_id, H, n_rep, kv, layer, scale, out);
}

cudaError_t trunk_init_attrs() {
    const cudaError_t e = set_smem_attrs(decode_attn_kernel, 0);
    return e != cudaSuccess ? e : set_smem_attrs(prefill_attn_kernel, PATTN_SMEM);
}

cudaError_t gather_rows_launch(const float* X, const int* src, const int* dst, int n, float* out,
                               int D, cudaStream_t s) {
    return launch(gather_rows_kernel, dim3(n), dim3(256), 0, s, false, X, src, dst, out, D);
}

// Argument checks of the decode-attention op (every pointer but the scratch).
int decode_attention_check(const float* qkv, int rows, int H, int KVH, int hd, const float* qn, const float* kn,
                           const float* rc, const float* rs, int max_len, const int32_t* pos, const float* kv_pool,
                           const int32_t* page_table, int max_pages, int page_size, int n_pages, int splits,
                           const float* out) {
    if (!qkv || !qn || !kn || !rc || !rs || !pos || !kv_pool || !page_table || !out)
        return fail(SKB_ERR_ARG, "decode_attention: null pointer");
    if (hd != 128 || KVH < 1 || H % KVH != 0 || H / KVH > 2)
        return fail(SKB_ERR_ARG, "decode_attention: head_dim must be 128 and heads/kv_heads 1 or 2");
    if (rows < 1 || rows > 65535 || max_len < 1 || max_pages < 1 || n_pages < 1 || splits < 1 || splits > 512)
        return fail(SKB_ERR_ARG, "decode_attention: bad sizes");
    if (page_size < 1 || (page_size & (page_size - 1)) != 0 || (long long)max_pages * page_size < max_len)
        return fail(SKB_ERR_ARG, "decode_attention: page_size must be a power of two covering max_len");
    // the kernels read these with 16-byte loads and bulk copies
    if (((uintptr_t)qkv | (uintptr_t)rc | (uintptr_t)rs | (uintptr_t)kv_pool | (uintptr_t)qn | (uintptr_t)kn) & 15u)
        return fail(SKB_ERR_ARG, "decode_attention: qkv, norm weights, RoPE tables and kv_pool must be 16-byte aligned");
    return SKB_OK;
}

int decode_attention_op(const float* qkv, int rows, int H, int KVH, int hd, const float* qn, const float* kn,
                        float eps, const float* rc, const float* rs, int max_len, const int32_t* pos, float* kv_pool,
                        const int32_t* page_table, int max_pages, int page_size, int n_pages, int splits,
                        float* part, int32_t* tickets, float* out, cudaStream_t stream) {
    const int chk = decode_attention_check(qkv, rows, H, KVH, hd, qn, kn, rc, rs, max_len, pos, kv_pool, page_table,
                                           max_pages, page_size, n_pages, splits, out);
    if (chk != SKB_OK) return chk;
    if (!part || !tickets) return fail(SKB_ERR_ARG, "decode_attention: null scratch pointer");
    DecodeAttnArgs a = {};
    a.qkv = qkv;
    a.ld_qkv = (H + 2 * KVH) * hd;
    a.qn = qn;
    a.kn = kn;
    a.eps = eps;
    a.rope_cos = rc;
    a.rope_sin = rs;
    a.pos = pos;
    a.max_len = max_len;
    a.kv.pool = kv_pool;
    a.kv.page_table = page_table;
    a.kv.max_pages = max_pages;
    int lg = 0;
    while ((1 << lg) < page_size) ++lg;
    a.kv.page_log2 = lg;
    a.kv.KVH = KVH;
    a.kv.hd = hd;
    a.kv.layer_floats = (long long)n_pages * 2 * KVH * page_size * hd;
    a.layer = 0;
    a.H = H;
    a.n_rep = H / KVH;
    a.S = splits;
    a.nmax = 0;
    a.scale = 1.0f / sqrtf((float)hd);
    a.part = part;
    a.counters = tickets;
    a.out = out;
    a.err = nullptr;
    a.kv.n_pages = n_pages;
    // up to 8 splits: one thread-block cluster per (row, kv head), merged in
    // distributed shared memory (the scratch is not touched); more splits:
    // partials in the caller's scratch, merged by the last CTA
    cudaError_t e = splits <= 8 ? decode_attn_cluster_launch(a, rows, stream, false)
                                : decode_attn_launch(a, rows, stream, false);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "decode_attention: %s", cudaGetErrorString(e));
}

}  // namespace skb

extern "C" int skb_test_gemm(const float* x, const float* w, float* out, int M, int N, int K, int tensor_cores,
                             int splits, cudaStream_t stream) {
    using namespace skb;
    if (!x || !w || !out || M < 1 || N < 1 || K < 32 || K % 32 != 0)
        return fail(SKB_ERR_ARG, "test_gemm: bad arguments (M=%d N=%d K=%d)", M, N, K);
    GemmArgs a = {};
    a.A = x;
    a.lda = K;
    a.w0 = w;
    a.seg1 = a.seg2 = 1 << 30;
    a.N = N;
    a.K = K;
    a.T = M;
    a.out = out;
    a.ldo = N;
    a.splits = splits;
    if (tensor_cores < 0 || tensor_cores > 3) return fail(SKB_ERR_ARG, "test_gemm: tensor_cores %d", tensor_cores);
    if (tensor_cores == 3 && (M > 32 || K % 256 != 0))
        return fail(SKB_ERR_ARG, "test_gemm: the FFMA kernel takes at most 32 rows and K % 256 == 0");
    a.variant = tensor_cores >= 2 ? tensor_cores - 1 : 0;
    const cudaError_t e = tensor_cores ? tgemm_launch(a, stream, false) : sgemm_launch(a, stream, false);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "test_gemm: %s", cudaGetErrorString(e));
}

extern "C" int skb_decode_attention(const float* qkv, int rows, int n_heads, int n_kv_heads, int head_dim,
                                    const float* q_norm, const float* k_norm, float eps, const float* rope_cos,
                                    const float* rope_sin, int max_len, const int32_t* pos, float* kv_pool,
                                    const int32_t* page_table, int max_pages, int page_size, int n_pages,
                                    int splits, float* part, int32_t* tickets, float* out, cudaStream_t stream) {
    return skb::decode_attention_op(qkv, rows, n_heads, n_kv_heads, head_dim, q_norm, k_norm, eps, rope_cos,
                                    rope_sin, max_len, pos, kv_pool, page_table, max_pages, page_size, n_pages,
                                    splits, part, tickets, out, stream);
}
