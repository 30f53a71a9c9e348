// Decode attention, one thread-block cluster per (row, kv head).
//
// Grid (C, KVH, R) with cluster dims (C, 1, 1), C <= 8.  CTA s of the cluster
// owns positions [s*T/C, (s+1)*T/C) of the row's T = p_new + 1 positions.
//
// Before the programmatic-dependent-launch wait -- everything it reads was
// written by kernels at least two launches back (the cache positions before
// p_new by earlier frames, the row position by the previous frame's last
// kernel) -- thread 0 looks up the pages of its range and stages the cached
// K and V rows into shared memory with 1-D bulk copies (TMA engine, one copy
// per page run, no multicast); the RoPE row of p_new and the q/k norm weights
// go to registers.  After the wait only the new q, k, v rows are read (one
// round trip).  Scores, softmax and P.V run on shared memory; the C partial
// (max, sum, output) triples are merged in split order by the cluster's rank
// 0 through distributed shared memory, so no global partials, atomics or
// second launch are needed.  Ranges longer than PMAX positions are processed
// in rounds with an online softmax.
//
// Two variants: for few (row, kv head) groups (batch-1 CFG: 16) a CTA stages
// 112 positions per round into one buffer (one CTA per SM, wide clusters);
// for many groups (batched rows) a CTA double-buffers rounds of 48 positions
// (two CTAs per SM), so the next round's copies overlap this round's math.
//
// (The merge area, ATC_MAXC partials, lives in rank 0's first K buffer.)
//
// Arithmetic restates transformers' Qwen3 attention step (modeling_qwen3.py:
// q_norm/k_norm :248-249, RoPE :130-181, GQA softmax :184-219, scaling
// head_dim**-0.5 :232).
#include "ops.cuh"
#include "trunk.cuh"
#include "trunk_api.cuh"

namespace skb {

constexpr int ATC_THREADS = 256;
constexpr int ATC_MAXC = 8;    // CTAs per cluster (portable cluster size)
constexpr int ATC_PART = 260;  // floats of one pushed partial: o[2][128], m[2], l[2]
// variants: (positions per round, buffers)
constexpr int ATC_PMAX_FEW = 112, ATC_NBUF_FEW = 1;
constexpr int ATC_PMAX_MANY = 48, ATC_NBUF_MANY = 2;
constexpr int ATC_MANY_GROUPS = 32;  // more (row, kv head) groups than this: the double-buffered variant

template <int PMAX, int NBUF>
struct AtcSmem {
    float k[NBUF][PMAX][128];
    float v[NBUF][PMAX][128];
    float q[2][128];
    float kn[128];
    float vn[128];
    float p[2][PMAX + 4];  // scores, then probabilities (+ the new position)
    float mr[2], lr[2];    // per-round block max / sum
    float wmx[8][2], wsm[8][2];  // double-buffered variant: per-round, per-warp score max / probability sum
    uint64_t bar[NBUF];
    uint64_t merge_bar;  // rank 0: every CTA's partial has arrived
    int err;
};
static_assert(ATC_MAXC * ATC_PART <= ATC_PMAX_MANY * 128, "merge area must fit in the K buffer");
static_assert(8 * 2 * 128 <= ATC_PMAX_MANY * 128, "warp sums must fit in the K buffer");

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Cluster barrier whose arrive orders no memory (relaxed) and whose wait
// acquires: the CTAs learn that every CTA finished reading its own shared
// memory, and see mbarriers initialised before a fence.mbarrier_init.
__device__ __forceinline__ void cluster_sync_exec() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Asynchronous store of a float into the shared memory of CTA `rank` of this
// cluster, completing (4 bytes of transaction count) on that CTA's mbarrier
// at the same offset as `bar`.
__device__ __forceinline__ void st_async_f32(float* p, float v, uint64_t* bar, uint32_t rank) {
    uint32_t rp, rb;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rp) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(smem_u32(bar)), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(rp),
                 "r"(__float_as_uint(v)), "r"(rb)
                 : "memory");
}

// Issues the bulk copies of cached positions [p0, p1) of (row r, head g)
// into buffer b of sm.k / sm.v (index = position - p0); returns the bytes
// requested.
template <int PMAX, int NBUF>
__device__ uint32_t atc_stage(const DecodeAttnArgs& a, int r, int g, int p0, int p1, AtcSmem<PMAX, NBUF>& sm,
                              int b) {
    uint32_t bytes = 0;
    const int page_sz = 1 << a.kv.page_log2;
    int p = p0;
    while (p < p1) {
        const int end = min(p1, ((p >> a.kv.page_log2) + 1) * page_sz);
        bytes += (uint32_t)(end - p) * 1024u;
        p = end;
    }
    if (bytes == 0) return 0;
    mbar_expect_tx(&sm.bar[b], bytes);
    p = p0;
    while (p < p1) {
        const int end = min(p1, ((p >> a.kv.page_log2) + 1) * page_sz);
        int page = __ldcg(a.kv.page_table + r * a.kv.max_pages + (p >> a.kv.page_log2));
        if ((unsigned)page >= (unsigned)a.kv.n_pages) page = 0;
        const int slot = p & (page_sz - 1);
        const float* kb = a.kv.pool + a.layer * a.kv.layer_floats +
                          ((((long long)page * 2 + 0) * a.kv.KVH + g) << a.kv.page_log2) * 128 + (long long)slot * 128;
        const float* vb = kb + ((long long)a.kv.KVH << a.kv.page_log2) * 128;
        const uint32_t nb = (uint32_t)(end - p) * 512u;
        bulk_g2s(&sm.k[b][p - p0][0], kb, nb, &sm.bar[b]);
        bulk_g2s(&sm.v[b][p - p0][0], vb, nb, &sm.bar[b]);
        p = end;
    }
    return bytes;
}

template <int PMAX, int NBUF>
__global__ void __launch_bounds__(ATC_THREADS) decode_attn_cluster_kernel(const DecodeAttnArgs a) {
    extern __shared__ __align__(128) unsigned char atc_raw[];
    AtcSmem<PMAX, NBUF>& sm = *reinterpret_cast<AtcSmem<PMAX, NBUF>*>(atc_raw);
    const int s = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int C = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_rep = a.n_rep;

    // debug stage times of this thread, flushed at the end so that no global
    // atomic sits before a barrier
    unsigned long long tl[7] = {0, 0, 0, 0, 0, 0, 0};
    if (tid == 0) {
        stamp_min(a.ts);
        for (int b = 0; b < NBUF; ++b) mbar_init(&sm.bar[b], 1);
        mbar_init(&sm.merge_bar, 1);
        mbar_fence_init();
        // rank 0 expects C partials of n_rep * (128 + 2) floats
        if (cluster_ctarank() == 0) mbar_expect_tx(&sm.merge_bar, (uint32_t)(C * n_rep * 130 * 4));
        sm.err = 0;
    }
    __syncthreads();

    // ---- before the wait: position, pages, cached K/V, RoPE row, norm weights
    int p_new = __ldcg(a.pos + r);
    const bool bad_pos = p_new < 0 || p_new >= a.max_len;
    if (bad_pos) p_new = p_new < 0 ? 0 : a.max_len - 1;
    const int T = p_new + 1;
    const int pb = (int)((long long)s * T / C);
    const int pe = (int)((long long)(s + 1) * T / C);
    const bool own_new = pe == T;            // the last CTA holds position p_new
    const int cend = own_new ? p_new : pe;   // cached positions [pb, cend)
    const int n_cached = cend > pb ? cend - pb : 0;
    const int n_rounds = n_cached > 0 ? (n_cached + PMAX - 1) / PMAX : 1;
    // copies issued / waited per buffer (thread 0's count): a buffer whose
    // last copy was not seen to land is waited on once more before exit
    int n_issued[NBUF], n_waited[NBUF];
#pragma unroll
    for (int b = 0; b < NBUF; ++b) n_issued[b] = n_waited[b] = 0;
    if (tid == 0) {
        for (int b = 0; b < NBUF && b < n_rounds; ++b) {
            const int p0 = pb + b * PMAX;
            if (atc_stage(a, r, g, p0, min(cend, p0 + PMAX), sm, b) > 0) ++n_issued[b];
        }
        // later rounds (long contexts) of the single-buffered variant: into
        // L2 now, into shared memory later.  The double-buffered variant
        // streams without it: its second buffer already keeps copies in
        // flight, and L2 prefetches running ahead of bulk copies slowed that
        // stream (92.4 against 97.9 us for 256 rows x 8 kv heads, measured)
        for (int p = pb + NBUF * PMAX; NBUF == 1 && p < cend;) {
            const int end = min(cend, ((p >> a.kv.page_log2) + 1) << a.kv.page_log2);
            const float* kb = a.kv.at(a.layer, r, p, 0, g);
            const float* vb = a.kv.at(a.layer, r, p, 1, g);
            bulk_prefetch_l2(kb, (unsigned)(end - p) * 512u);
            bulk_prefetch_l2(vb, (unsigned)(end - p) * 512u);
            p = end;
        }
    }
    const float* cosr = a.rope_cos + (size_t)p_new * 64;
    const float* sinr = a.rope_sin + (size_t)p_new * 64;
    // cache slots of p_new (the page lookup is done before the wait too)
    float* kdst = (own_new && warp == 2) ? a.kv.at(a.layer, r, p_new, 0, g) : nullptr;
    float* vdst = (own_new && warp == 3) ? a.kv.at(a.layer, r, p_new, 1, g) : nullptr;

    pdl_wait();
    if (tid == 0) stamp_wait(a.ts);
    if (tid == 0 && bad_pos && a.err != nullptr) atomicExch(a.err, 1);

    // ---- the new q (n_rep heads), k and v of this kv head: one round trip
    const float* row = a.qkv + (size_t)r * a.ld_qkv;
    if (warp < n_rep) {
        const int h = g * n_rep + warp;
        float4 q = ld_cg4(reinterpret_cast<const float4*>(row + h * 128) + lane);
        q = norm_rope_head(q, a.qn, a.eps, cosr, sinr, lane, true, true);
        q.x *= a.scale;
        q.y *= a.scale;
        q.z *= a.scale;
        q.w *= a.scale;
        reinterpret_cast<float4*>(sm.q[warp])[lane] = q;
    } else if (warp == 2) {
        float4 k = ld_cg4(reinterpret_cast<const float4*>(row + (a.H + g) * 128) + lane);
        k = norm_rope_head(k, a.kn, a.eps, cosr, sinr, lane, true, true);
        reinterpret_cast<float4*>(sm.kn)[lane] = k;
        if (kdst) reinterpret_cast<float4*>(kdst)[lane] = k;
    } else if (warp == 3) {
        const float4 v = ld_cg4(reinterpret_cast<const float4*>(row + (a.H + a.kv.KVH + g) * 128) + lane);
        reinterpret_cast<float4*>(sm.vn)[lane] = v;
        if (vdst) reinterpret_cast<float4*>(vdst)[lane] = v;
    }
    pdl_trigger();
    __syncthreads();
    tl[0] = a.ts ? globaltimer_ns() : 0;

    // ---- rounds of up to PMAX cached positions (+ p_new in the last)
    // Scores: lane 8G+t of a warp works on slot i0+G and float4 columns
    // t, t+8, t+16, t+24 of the K row (each 8-lane phase of a 128-bit shared
    // load reads 128 contiguous bytes: no bank conflicts), reduced over the
    // 8 lanes by 3 shuffles.  P.V: warp gp accumulates slots i = gp mod 8 for
    // both heads (lane pc: float4 column pc), so each V row is read once; the
    // 8 warps' sums are added in warp order at the end.
    const int sg = lane >> 3, st8 = lane & 7;
    float4 qa[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            qa[h][j] = reinterpret_cast<const float4*>(sm.q[h < n_rep ? h : 0])[st8 + 8 * j];
    const int pc = lane, gp = warp;
    float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    for (int rd = 0; rd < n_rounds; ++rd) {
        // a copy that timed out stops the rounds (sm.err was written before
        // the last barrier, so every thread takes the same branch)
        if (sm.err) break;
        const int b = rd % NBUF;
        const int r0 = pb + rd * PMAX;
        const int nc = max(0, min(PMAX, cend - r0));  // cached positions this round
        const bool last = rd == n_rounds - 1;
        const int ns = nc + ((last && own_new) ? 1 : 0);  // score slots
        if (NBUF == 1 && rd > 0 && tid == 0 && atc_stage(a, r, g, r0, r0 + nc, sm, 0) > 0) ++n_issued[0];
        if (nc > 0) {
            // the round's copy is use number rd / NBUF of its buffer
            if (!mbar_wait(&sm.bar[b], (uint32_t)(rd / NBUF) & 1u, a.err)) sm.err = 1;
            ++n_waited[b];
        }
        if (rd == 0) tl[1] = a.ts ? globaltimer_ns() : 0;
        float wm0 = -INFINITY, wm1 = -INFINITY;  // this warp's score max per head (double-buffered variant)
        for (int i0 = warp * 4; i0 < ns; i0 += 32) {
            const int i = i0 + sg;
            const float4* kr = reinterpret_cast<const float4*>(i < nc ? sm.k[b][i < nc ? i : 0] : sm.kn);
            float s0 = 0.f, s1 = 0.f;
            if (i < ns) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 kv = kr[st8 + 8 * j];
                    s0 = fmaf(qa[0][j].x, kv.x, s0);
                    s0 = fmaf(qa[0][j].y, kv.y, s0);
                    s0 = fmaf(qa[0][j].z, kv.z, s0);
                    s0 = fmaf(qa[0][j].w, kv.w, s0);
                    s1 = fmaf(qa[1][j].x, kv.x, s1);
                    s1 = fmaf(qa[1][j].y, kv.y, s1);
                    s1 = fmaf(qa[1][j].z, kv.z, s1);
                    s1 = fmaf(qa[1][j].w, kv.w, s1);
                }
            }
#pragma unroll
            for (int o = 4; o >= 1; o >>= 1) {
                s0 += __shfl_xor_sync(FULL, s0, o);
                s1 += __shfl_xor_sync(FULL, s1, o);
            }
            if (st8 == 0 && i < ns) {
                sm.p[0][i] = s0;
                if (n_rep > 1) sm.p[1][i] = s1;
            }
            if (NBUF > 1 && i < ns) {
                wm0 = fmaxf(wm0, s0);
                wm1 = fmaxf(wm1, s1);
            }
        }
        if constexpr (NBUF > 1) {
            wm0 = warp_max(wm0);
            wm1 = warp_max(wm1);
            if (lane == 0) {
                sm.wmx[warp][0] = wm0;
                sm.wmx[warp][1] = wm1;
            }
        }
        __syncthreads();
        if (rd == 0) tl[2] = a.ts ? globaltimer_ns() : 0;
        if constexpr (NBUF > 1) {
            // the round's max per head (warps in order); every warp turns its
            // own slots into probabilities: lane l takes head l / 16 and the
            // warp's slot number l % 16 (slots warp*4 + 32k + j, k, j < 4)
            static_assert(PMAX + 1 <= 128, "16 lanes per head cover a warp's slots only below 128");
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                mx0 = fmaxf(mx0, sm.wmx[w][0]);
                mx1 = fmaxf(mx1, sm.wmx[w][1]);
            }
            const float mn0 = fmaxf(m_run[0], mx0), mn1 = n_rep > 1 ? fmaxf(m_run[1], mx1) : -INFINITY;
            const int h = lane >> 4, t = lane & 15;
            const int i = warp * 4 + 32 * (t >> 2) + (t & 3);
            const float mh = h == 0 ? mn0 : mn1;
            float e = 0.f;
            if (h < n_rep && i < ns) {
                e = (mh == -INFINITY) ? 0.f : expf(sm.p[h][i] - mh);
                sm.p[h][i] = e;
            }
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) e += __shfl_xor_sync(FULL, e, o);  // within each half-warp
            if (t == 0) sm.wsm[warp][h] = e;
            __syncthreads();
            if (tid < 2) {  // the round's (max, sum) per head, sums in warp order
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) sum += sm.wsm[w][tid];
                sm.mr[tid] = tid == 0 ? mn0 : mn1;
                sm.lr[tid] = sum;
            }
        } else if (warp < n_rep) {
            // per-head max (warp h), then probabilities and their sum (warp h)
            float mx = -INFINITY;
            for (int i = lane; i < ns; i += 32) mx = fmaxf(mx, sm.p[warp][i]);
            mx = warp_max(mx);
            const float mnew = fmaxf(m_run[warp], mx);
            float sum = 0.f;
            for (int i = lane; i < ns; i += 32) {
                const float e = (mnew == -INFINITY) ? 0.f : expf(sm.p[warp][i] - mnew);
                sm.p[warp][i] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                sm.mr[warp] = mnew;
                sm.lr[warp] = sum;
            }
        }
        __syncthreads();
        if (rd == 0) tl[3] = a.ts ? globaltimer_ns() : 0;
        // online update of (m, l, o) and P.V over this round's slots
        float corr[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float mnew = h < n_rep ? sm.mr[h] : -INFINITY;
            corr[h] = (m_run[h] == -INFINITY) ? 0.f : expf(m_run[h] - mnew);
            l_run[h] = l_run[h] * corr[h] + (h < n_rep ? sm.lr[h] : 0.f);
            m_run[h] = mnew;
        }
        {
            const float c0 = corr[0], c1 = corr[1];
            acc0 = make_float4(acc0.x * c0, acc0.y * c0, acc0.z * c0, acc0.w * c0);
            acc1 = make_float4(acc1.x * c1, acc1.y * c1, acc1.z * c1, acc1.w * c1);
            for (int i = gp; i < ns; i += 8) {
                const float p0 = sm.p[0][i];
                const float p1 = n_rep > 1 ? sm.p[1][i] : 0.f;
                const float4 vv = reinterpret_cast<const float4*>(i < nc ? sm.v[b][i < nc ? i : 0] : sm.vn)[pc];
                acc0.x = fmaf(p0, vv.x, acc0.x);
                acc0.y = fmaf(p0, vv.y, acc0.y);
                acc0.z = fmaf(p0, vv.z, acc0.z);
                acc0.w = fmaf(p0, vv.w, acc0.w);
                acc1.x = fmaf(p1, vv.x, acc1.x);
                acc1.y = fmaf(p1, vv.y, acc1.y);
                acc1.z = fmaf(p1, vv.z, acc1.z);
                acc1.w = fmaf(p1, vv.w, acc1.w);
            }
        }
        __syncthreads();  // sm.k / sm.v / sm.p are refilled by the next round
        // double buffering: this buffer takes round rd + NBUF
        if (NBUF > 1 && tid == 0 && rd + NBUF < n_rounds) {
            const int q0 = pb + (rd + NBUF) * PMAX;
            if (atc_stage(a, r, g, q0, min(cend, q0 + PMAX), sm, b) > 0) ++n_issued[b];
        }
    }
    // the 8 warps' sums, added in warp order (K buffer as scratch)
    float* gsum = &sm.k[0][0][0];  // [8][2][128]
    reinterpret_cast<float4*>(gsum + (gp * 2 + 0) * 128)[pc] = acc0;
    reinterpret_cast<float4*>(gsum + (gp * 2 + 1) * 128)[pc] = acc1;
    __syncthreads();
    const int hh = tid >> 7, d = tid & 127;  // merge: thread (head hh, dim d)
    float o_run = 0.f;
    if (hh < n_rep) {
#pragma unroll
        for (int w = 0; w < 8; ++w) o_run += gsum[(w * 2 + hh) * 128 + d];
    }
    tl[4] = a.ts ? globaltimer_ns() : 0;

    // ---- merge: once every CTA of the cluster is done with its K/V buffers
    // (an execution-only cluster barrier, which also publishes rank 0's merge
    // barrier initialised at the start), each sends its partial (output, max,
    // sum) into rank 0's K buffer with asynchronous remote stores that count
    // down rank 0's merge barrier; rank 0 merges them in split order.
    if (tid == 0 && sm.err) {
        // a copy did not arrive in time: flag it and wait (bounded) once more
        // on every buffer's last copy so that none is still in flight when
        // the buffers are reused
        if (a.err != nullptr) atomicExch(a.err, 1);
#pragma unroll
        for (int b = 0; b < NBUF; ++b)
            if (n_issued[b] > 0) mbar_wait(&sm.bar[b], (uint32_t)(n_issued[b] - 1) & 1u, nullptr);
    }
    __syncthreads();  // the group sums in the K buffer are read
    cluster_sync_exec();
    tl[5] = a.ts ? globaltimer_ns() : 0;
    const uint32_t rank = cluster_ctarank();
    float* slot = &sm.k[0][0][0] + (size_t)rank * ATC_PART;  // [2][128] o | [2] m | [2] l
    if (hh < n_rep) {
        st_async_f32(slot + hh * 128 + d, o_run, &sm.merge_bar, 0);
        if (d == 0) {
            st_async_f32(slot + 256 + hh, m_run[hh], &sm.merge_bar, 0);
            st_async_f32(slot + 258 + hh, l_run[hh], &sm.merge_bar, 0);
        }
    }
    if (rank == 0 && hh < n_rep) {
        const bool ok = mbar_wait(&sm.merge_bar, 0, a.err);
        tl[6] = a.ts ? globaltimer_ns() : 0;
        if (ok) {
            const float* parts = &sm.k[0][0][0];
            float M = -INFINITY;
            for (int j = 0; j < C; ++j) M = fmaxf(M, parts[j * ATC_PART + 256 + hh]);
            float L = 0.f, O = 0.f;
            for (int j = 0; j < C; ++j) {
                const float* pj = parts + j * ATC_PART;
                const float mj = pj[256 + hh];
                const float w = (mj == -INFINITY) ? 0.f : expf(mj - M);
                L = fmaf(pj[258 + hh], w, L);
                O = fmaf(pj[hh * 128 + d], w, O);
            }
            a.out[(size_t)r * a.H * 128 + (g * n_rep + hh) * 128 + d] = O / L;
        }
    }
    // rank 0 arrives once every partial has landed, so no CTA exits with one
    // of its remote stores still in flight
    cluster_sync_exec();
    if (a.ts) {
        __syncthreads();
        if (tid == 0) {
            stamp_max(a.ts + 3);
#pragma unroll
            for (int k = 0; k < 7; ++k) atomicMax(a.ts + 4 + k, tl[k]);
        }
    }
}

using AtcFew = AtcSmem<ATC_PMAX_FEW, ATC_NBUF_FEW>;
using AtcMany = AtcSmem<ATC_PMAX_MANY, ATC_NBUF_MANY>;
#define ATC_KERNEL_FEW decode_attn_cluster_kernel<ATC_PMAX_FEW, ATC_NBUF_FEW>
#define ATC_KERNEL_MANY decode_attn_cluster_kernel<ATC_PMAX_MANY, ATC_NBUF_MANY>

cudaError_t decode_attn_cluster_prepare() {
    cudaError_t e = set_smem_attrs(ATC_KERNEL_FEW, sizeof(AtcFew));
    if (e == cudaSuccess) e = set_smem_attrs(ATC_KERNEL_MANY, sizeof(AtcMany));
    return e;
}

// Widest cluster (<= 8 CTAs) for which `groups` clusters can be resident at
// once on this GPU (a cluster's CTAs must share one GPC; with ~119 KB of shared
// memory per CTA a B200 holds 15 clusters of 8 but needs 16 at bs1 CFG).
int decode_attn_cluster_width(int groups) {
    if (decode_attn_cluster_prepare() != cudaSuccess) {
        cudaGetLastError();
        return 1;
    }
    const bool many = groups > ATC_MANY_GROUPS;
    for (int c = ATC_MAXC; c > 1; --c) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c, 1, 1);
        cfg.blockDim = dim3(ATC_THREADS);
        cfg.dynamicSmemBytes = many ? sizeof(AtcMany) : sizeof(AtcFew);
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = c;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t e = many ? cudaOccupancyMaxActiveClusters(&n, ATC_KERNEL_MANY, &cfg)
                                   : cudaOccupancyMaxActiveClusters(&n, ATC_KERNEL_FEW, &cfg);
        if (e != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (n >= groups) return c;
    }
    return 1;
}

// C = a.S CTAs per (row, kv head), 1 <= C <= 8; head_dim 128, n_rep <= 2.
// a.variant 0 picks the double-buffered kernel for more than 32 (row, kv
// head) groups; a caller whose batch width varies fixes it (1 / 2) so that a
// row's arithmetic does not depend on how many rows run beside it.
cudaError_t decode_attn_cluster_launch(const DecodeAttnArgs& a, int R, cudaStream_t s, bool pdl) {
    static bool prepared = false;
    if (!prepared) {
        const cudaError_t e = decode_attn_cluster_prepare();
        if (e != cudaSuccess) return e;
        prepared = true;
    }
    if (a.S < 1 || a.S > ATC_MAXC || a.n_rep < 1 || a.n_rep > 2 || a.kv.hd != 128) return cudaErrorInvalidValue;
    const bool many = a.variant == 0 ? R * a.kv.KVH > ATC_MANY_GROUPS : a.variant == 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.S, a.kv.KVH, R);
    cfg.blockDim = dim3(ATC_THREADS);
    cfg.dynamicSmemBytes = many ? sizeof(AtcMany) : sizeof(AtcFew);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return many ? cudaLaunchKernelEx(&cfg, ATC_KERNEL_MANY, a) : cudaLaunchKernelEx(&cfg, ATC_KERNEL_FEW, a);
}

}  // namespace skb
