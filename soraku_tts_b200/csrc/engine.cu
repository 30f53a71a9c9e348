// Decode engine: the GraphFrameEngine replacement (graph_frame.py:23-328).
//
// One frame (graph_frame.py:201-272) is 16 depth steps followed by one trunk
// step; on the GPU it is a fixed list of kernels:
//
//   for q in 0..15:
//     D_up(q)     a = rmsnorm_in(rmsnorm_final(x) + prefix); act = silu(a Wg^T) * (a Wu^T)
//     D_down(q)   y = act Wd^T + a
//     D_cls(q)    logits = rmsnorm_out(y) table[q]^T + bias[q]
//     D_samp(q)   CFG + mask + temperature + top-k/top-p + Philox draw -> code;
//                 prefix += table[q][code] * scale   (q = 15: x = frame embedding)
//   for l in 0..L-1:
//     QKV(l)      qkv = rmsnorm(x) [Wq;Wk;Wv]^T
//     ATTN(l)     q/k norm, RoPE, KV append, split-K GQA attention (+ combine)
//     O(l)        x += attn Wo^T
//     GU(l)       act = silu(n Wg^T) * (n Wu^T),  n = rmsnorm(x)
//     DOWN(l)     x += act Wd^T                   (l = L-1: pos += 1)
//
// x holds the pre-final-norm residual stream of each CFG row; the final norm
// is folded into D_up's prologue.  Kernels are chained with programmatic
// dependent launch, and each kernel bulk-prefetches the next kernel's weights
// into L2 before waiting on its predecessor, so HBM keeps streaming across
// kernel boundaries.  The list is recorded once as a CUDA graph.
#include <cmath>
#include <cstring>
#include <functional>
#include <vector>

#include "depth_head.cuh"
#include "engine_types.cuh"
#include "trunk.cuh"
#include "ops.cuh"
#include "sampler.cuh"
#include "trunk_api.cuh"

namespace skb {

// VMAX: audio vocabulary capacity (2304 covers soraku's 2051 codes with 9
// logits per thread).
template <int VMAX>
__global__ void __launch_bounds__(SAMPLER_THREADS) depth_sample_kernel(const DepthSampleArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int codes_s[32];
    if (threadIdx.x == 0) stamp_min(a.ts);
    prefetch_share(a.pf, blockIdx.x, gridDim.x);
    int frame;
    const SampleJob J = depth_sample_job(a, blockIdx.x, &frame);
    pdl_wait();
    if (threadIdx.x == 0) stamp_wait(a.ts);
    pdl_trigger();
    depth_sample_body<BlockSync, VMAX>(a, blockIdx.x, J, frame, smem, codes_s);
    if (a.ts) {
        __syncthreads();
        if (threadIdx.x == 0) stamp_max(a.ts + 3);
    }
}

}  // namespace skb

using namespace skb;

struct skb_engine {
    skb_model_desc m;
    std::vector<const float*> lw;  // layer pointers
    skb_engine_opts o;
    int device = 0, nsm = 148;
    int R = 0, rpr = 1, nreq = 0;
    int D = 0, H = 0, KVH = 0, hd = 0, F = 0, I = 0, Q = 0, V = 0, L = 0, n_rep = 1;
    int max_pages = 0, page_log2 = 6, S = 1;
    long long layer_floats = 0;
    // decode state
    float *x = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *abuf = nullptr, *y = nullptr,
          *hidden = nullptr, *logits = nullptr, *logits_hist = nullptr, *prefix = nullptr,
          *rope_cos = nullptr, *rope_sin = nullptr, *kv = nullptr;
    int *pos = nullptr, *page_table = nullptr, *err = nullptr, *host_flag = nullptr;
    int64_t *cur_codes = nullptr, *hist = nullptr;
    ReqState* st = nullptr;
    // prefill scratch
    float *pX = nullptr, *pN = nullptr, *pQKV = nullptr, *pQ = nullptr, *pA = nullptr, *pG = nullptr,
          *spk = nullptr, *spk_in = nullptr;
    PrefillTok* ptok = nullptr;
    int64_t* pframes = nullptr;
    int* pmeta = nullptr;  // [5][prefill rows]: row_off | row_len | row_id | gather_src | gather_dst
    int prefill_batch = 1;  // requests one prefill pass can hold
    // graph
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    int graph_active = 0, graph_fpg = 0, graph_pdl = 0;
    // captured graphs by (batch width, frames per replay), least recently used evicted
    struct CachedGraph {
        int n_active, fpg, pdl;
        cudaGraphExec_t exec;
        unsigned long long used;
    };
    std::vector<CachedGraph> graphs;
    unsigned long long graph_clock = 0;
    int debug = 0;
    float* xn = nullptr;  // batched path: normalised activations [R][max inner size]
    int gemm_min_rows = 5;  // batches of at least this many rows take the tensor-core GEMM path
    int attn_variant = 1;   // cluster attention kernel (fixed per engine: see DecodeAttnArgs::variant)
    int* pt_tmp = nullptr;  // page-table row scratch for move_request
    int pool_pages = 0;     // KV pages per layer
    bool shared_pool = false;  // pages mapped by the caller (skb_engine_map_pages)
    std::vector<int> pt_host;  // host mirror of the page table
    int frame_nodes = 0;  // kernels of the last built frame
    unsigned long long* kts = nullptr;  // debug kernel timeline [kernels per frame][SKB_KTS_STRIDE]
    std::vector<int> frames_host, pos_host;
    std::vector<ReqState> st_host;
    std::vector<void*> allocs;
    // device error flags seen from the host: each step queues a copy of the
    // flags into pinned memory; a later step checks it once it has landed
    // persistent depth head (depth_head.cu) for a batch of one CFG request
    bool dh_ok = false;
    unsigned* dh_bar = nullptr;  // its grid barrier word
    int* dh_abort = nullptr;
    unsigned long long* dh_ts = nullptr;  // debug phase timeline [4 Q][2]
    int* err_host = nullptr;
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;
    int err_seen = -1;  // index of the first raised flag observed (sticky)
};

namespace {

enum : int { PH_GEMV = 0, PH_ATTN = 1 };

// One step of the frame program: a GEMV launch (whose classifier step may
// carry the depth sampler that follows it) or a decode-attention launch.
struct Phase {
    int kind;
    int xm, em;
    int pre_normed;  // batched rows: the previous sampler wrote this phase's normed rows
    int sample;
    int n_req;
    GemvArgs g;
    DepthSampleArgs s;
    DecodeAttnArgs at;
};

template <typename T>
int dalloc(skb_engine* e, T** p, size_t n) {
    void* ptr = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&ptr, n * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(SKB_ERR_NOMEM, "cudaMalloc of %zu bytes failed", n * sizeof(T));
    }
    cudaMemset(ptr, 0, n * sizeof(T));
    e->allocs.push_back(ptr);
    *p = reinterpret_cast<T*>(ptr);
    return SKB_OK;
}

KVLayout kv_layout(const skb_engine* e) {
    KVLayout k;
    k.pool = e->kv;
    k.page_table = e->page_table;
    k.max_pages = e->max_pages;
    k.page_log2 = e->page_log2;
    k.KVH = e->KVH;
    k.hd = e->hd;
    k.layer_floats = e->layer_floats;
    k.n_pages = e->pool_pages;
    return k;
}

const float* LW(const skb_engine* e, int l, int which) { return e->lw[(size_t)l * SKB_LAYER_PTRS + which]; }
enum { W_Q = 0, W_K, W_V, W_O, W_QN, W_KN, W_G, W_U, W_D, W_LN1, W_LN2 };

struct WRange {
    const char* p;
    unsigned long long bytes;
};

// One kernel of the frame: its launcher (given the prefetch list of the next
// kernel's weights) and the weight ranges it reads.
struct Node {
    std::vector<WRange> w;
    int ctas = 0;  // CTAs of the launch; only wide kernels issue L2 prefetches
    std::function<cudaError_t(cudaStream_t, bool, const PrefetchList&)> run;
};

std::vector<WRange> gemv_ranges(const GemvArgs& a) {
    std::vector<WRange> r;
    const unsigned long long rowb = (unsigned long long)a.K * 4;
    if (a.interleave) {
        r.push_back({(const char*)a.w0, rowb * (a.N / 2)});
        r.push_back({(const char*)a.w1, rowb * (a.N / 2)});
    } else {
        const int s1 = a.seg1 < a.N ? a.seg1 : a.N;
        const int s2 = a.seg2 < a.N ? a.seg2 : a.N;
        r.push_back({(const char*)a.w0, rowb * s1});
        if (s2 > s1) r.push_back({(const char*)a.w1, rowb * (s2 - s1)});
        if (a.N > s2) r.push_back({(const char*)a.w2, rowb * (a.N - s2)});
    }
    return r;
}

Node gemv_node(const skb_engine* e, GemvArgs a, int M, int XM, int EM) {
    Node n;
    n.w = gemv_ranges(a);
    a.err = e->err + 2;
    const int units = a.N / (EM == E_SWIGLU ? 2 : 1);
    const int grid = units < e->nsm ? units : e->nsm;
    n.ctas = grid;
    n.run = [a, M, XM, EM, grid](cudaStream_t s, bool pdl, const PrefetchList& pf) {
        GemvArgs b = a;
        b.pf = pf;
        return gemv_launch(b, M, XM, EM, grid, s, pdl);
    };
    return n;
}

Phase gemv_phase(const GemvArgs& a, int XM, int EM) {
    Phase ph = {};
    ph.kind = PH_GEMV;
    ph.xm = XM;
    ph.em = EM;
    ph.g = a;
    return ph;
}

// The frame as a program of phases (16 depth steps, then the trunk layers),
// turned into kernel launches chained with PDL by build_frame.
// Debug timeline blocks: at most 6 launches per depth step (norm + GEMM for
// up and classifier, down, sampler), 7 per layer (norm + GEMM for QKV and
// gate/up, attention, O, down) and the position advance.
int kts_slots(const skb_engine* e) { return e->Q * 6 + e->L * 7 + 1; }
unsigned long long* node_stamps(const skb_engine* e, size_t node) {
    return (e->debug && (int)node < kts_slots(e)) ? e->kts + SKB_KTS_STRIDE * node : nullptr;
}

std::vector<Phase> build_phases(skb_engine* e, int n_active) {
    std::vector<Phase> phases;
    const int R = n_active * e->rpr;
    const int D = e->D;
    for (int q = 0; q < e->Q; ++q) {
        float* lg = e->debug ? e->logits_hist + (size_t)q * e->R * e->V : e->logits;
        {  // D_up
            GemvArgs a = gemv_args_plain(e->x, D, 2 * e->I, D);
            a.w0 = e->m.depth_gate;
            a.w1 = e->m.depth_up;
            a.interleave = 1;
            a.nw2 = e->m.final_norm;
            a.neps2 = e->m.rms_eps;
            a.x2 = e->prefix;
            a.ldx2 = D;
            a.x2_div = e->rpr;
            a.nw = e->m.depth_norm_in;
            a.neps = e->m.depth_eps;
            a.xout = e->abuf;
            a.hout = e->hidden;
            a.out = e->act;
            a.ldo = e->I;
            phases.push_back(gemv_phase(a, X_NORM_ADD_NORM, E_SWIGLU));
            phases.back().pre_normed = (R >= e->gemm_min_rows && q > 0 && D <= 1024) ? 1 : 0;
        }
        {  // D_down
            GemvArgs a = gemv_args_plain(e->act, e->I, D, e->I);
            a.w0 = e->m.depth_down;
            a.resid = e->abuf;
            a.ldr = D;
            a.out = e->y;
            a.ldo = D;
            phases.push_back(gemv_phase(a, X_PLAIN, E_RESID));
        }
        {  // D_cls
            GemvArgs a = gemv_args_plain(e->y, D, e->V, D);
            a.w0 = e->m.table + (size_t)q * e->V * D;
            a.nw = e->m.depth_norm_out;
            a.neps = e->m.depth_eps;
            a.bias = e->m.depth_bias + (size_t)q * e->V;
            a.out = lg;
            a.ldo = e->V;
            phases.push_back(gemv_phase(a, X_RMSNORM, E_BIAS));
        }
        {  // D_samp: the classifier phase's sampler
            DepthSampleArgs a = {};
            a.logits = lg;
            a.rows_per_req = e->rpr;
            a.V = e->V;
            a.q = q;
            a.Q = e->Q;
            a.D = D;
            a.st = e->st;
            a.host_flag = e->host_flag;
            a.table = e->m.table;
            a.scale = e->m.frame_scale;
            a.prefix = e->prefix;
            a.x = e->x;
            a.cur_codes = e->cur_codes;
            a.hist = e->hist;
            a.max_frames = e->o.max_frames;
            a.bos = e->m.bos_id;
            a.pad = e->m.pad_id;
            a.eos = e->m.eos_id;
            // batched rows: the sampler also forms the next step's depth
            // input rows (replacing that step's row-norm launch)
            if (R >= e->gemm_min_rows && q < e->Q - 1 && D <= 1024) {
                a.fn_w = e->m.final_norm;
                a.fn_eps = e->m.rms_eps;
                a.ni_w = e->m.depth_norm_in;
                a.ni_eps = e->m.depth_eps;
                a.xn = e->xn;
                a.xout = e->abuf;
                a.hout = e->hidden;
            }
            Phase& cls = phases.back();
            cls.sample = 1;
            cls.n_req = n_active;
            cls.s = a;
        }
    }
    const int qd = e->H * e->hd, kvd = e->KVH * e->hd;
    for (int l = 0; l < e->L; ++l) {
        {  // QKV
            GemvArgs a = gemv_args_plain(e->x, D, qd + 2 * kvd, D);
            a.w0 = LW(e, l, W_Q);
            a.w1 = LW(e, l, W_K);
            a.w2 = LW(e, l, W_V);
            a.seg1 = qd;
            a.seg2 = qd + kvd;
            a.nw = LW(e, l, W_LN1);
            a.neps = e->m.rms_eps;
            a.out = e->qkv;
            a.ldo = qd + 2 * kvd;
            phases.push_back(gemv_phase(a, X_RMSNORM, E_STORE));
        }
        {  // ATTN
            DecodeAttnArgs a = {};
            a.qkv = e->qkv;
            a.ld_qkv = qd + 2 * kvd;
            a.qn = LW(e, l, W_QN);
            a.kn = LW(e, l, W_KN);
            a.eps = e->m.rms_eps;
            a.rope_cos = e->rope_cos;
            a.rope_sin = e->rope_sin;
            a.pos = e->pos;
            a.max_len = e->o.max_len;
            a.kv = kv_layout(e);
            a.layer = l;
            a.H = e->H;
            a.n_rep = e->n_rep;
            a.S = e->S;
            a.variant = e->attn_variant;
            a.scale = 1.0f / sqrtf((float)e->hd);
            a.out = e->attn;
            a.err = e->err;
            Phase ph = {};
            ph.kind = PH_ATTN;
            ph.at = a;
            phases.push_back(ph);
        }
        {  // O
            GemvArgs a = gemv_args_plain(e->attn, qd, D, qd);
            a.w0 = LW(e, l, W_O);
            a.resid = e->x;
            a.ldr = D;
            a.out = e->x;
            a.ldo = D;
            phases.push_back(gemv_phase(a, X_PLAIN, E_RESID));
        }
        {  // GU
            GemvArgs a = gemv_args_plain(e->x, D, 2 * e->F, D);
            a.w0 = LW(e, l, W_G);
            a.w1 = LW(e, l, W_U);
            a.interleave = 1;
            a.nw = LW(e, l, W_LN2);
            a.neps = e->m.rms_eps;
            a.out = e->act;
            a.ldo = e->F;
            phases.push_back(gemv_phase(a, X_RMSNORM, E_SWIGLU));
        }
        {  // DOWN
            GemvArgs a = gemv_args_plain(e->act, e->F, D, e->F);
            a.w0 = LW(e, l, W_D);
            a.resid = e->x;
            a.ldr = D;
            a.out = e->x;
            a.ldo = D;
            if (l == e->L - 1) {
                a.inc = e->pos;
                a.n_inc = R;
            }
            phases.push_back(gemv_phase(a, X_PLAIN, E_RESID));
        }
    }
    return phases;
}

// Separate kernels: one GEMV launch per GEMV phase (+ the sampler after the
// classifier), one attention launch per attention phase.
// Batched rows (more than the ring GEMV's 4): the phase as a row-norm kernel
// (when its prologue normalises) and the 3xTF32 tensor-core GEMM over all
// rows, then the position advance of the frame's last GEMV.
void gemm_rows_nodes(skb_engine* e, const Phase& ph, int R, std::vector<Node>& nodes) {
    const GemvArgs& g = ph.g;
    if (ph.xm != X_PLAIN && !ph.pre_normed) {
        NormRowsArgs na = {};
        na.x = g.x;
        na.ldx = g.ldx;
        na.x2 = g.x2;
        na.ldx2 = g.ldx2;
        na.x2_div = g.x2_div > 0 ? g.x2_div : 1;
        na.nw = g.nw;
        na.eps = g.neps;
        na.nw2 = g.nw2;
        na.eps2 = g.neps2;
        na.xn = e->xn;
        na.xout = g.xout;
        na.hout = g.hout;
        na.D = g.K;
        na.mode = ph.xm == X_NORM_ADD_NORM ? 3 : 1;
        na.ts = node_stamps(e, nodes.size());
        Node n;
        n.ctas = R;
        n.run = [na, R](cudaStream_t s, bool pdl, const PrefetchList&) {
            return norm_rows(na, R, s, pdl) == SKB_OK ? cudaSuccess : cudaErrorUnknown;
        };
        nodes.push_back(n);
    }
    GemmArgs a = {};
    a.A = ph.xm == X_PLAIN ? g.x : e->xn;
    a.lda = ph.xm == X_PLAIN ? g.ldx : g.K;
    a.w0 = g.w0;
    a.w1 = g.w1;
    a.w2 = g.w2;
    a.seg1 = g.seg1;
    a.seg2 = g.seg2;
    a.interleave = g.interleave;
    a.N = g.N;
    a.K = g.K;
    a.T = R;
    a.out = g.out;
    a.ldo = g.ldo;
    a.resid = g.resid;
    a.ldr = g.ldr;
    a.bias = g.bias;
    a.mode = ph.em == E_RESID ? 1 : (ph.em == E_BIAS ? 2 : (ph.em == E_SWIGLU ? 3 : 0));
    a.err = e->err + 2;
    a.ts = node_stamps(e, nodes.size());
    Node n;
    n.w = gemv_ranges(g);
    n.ctas = ((a.N + 63) / 64) * ((R + 127) / 128);
    n.run = [a](cudaStream_t s, bool pdl, const PrefetchList&) { return tgemm_launch(a, s, pdl); };
    nodes.push_back(n);
    if (g.inc != nullptr) {
        int* inc = g.inc;
        const int n_inc = g.n_inc;
        Node adv;
        adv.ctas = 1;
        adv.run = [inc, n_inc](cudaStream_t s, bool pdl, const PrefetchList&) {
            return advance_launch(inc, n_inc, s, pdl);
        };
        nodes.push_back(adv);
    }
}

// The frame's kernel list for a batch of n_active requests.  A captured graph
// bakes in, besides n_active and frames per replay (its cache key), engine
// state fixed at creation: the buffers and weight pointers, gemm_min_rows,
// attn_variant, the attention split count S, the opts' use_pdl and
// l2_prefetch, and the debug flag.  skb_engine_set_debug drops every cached
// graph when the flag changes; any future setter of the other state must do
// the same (destroy_graph) or add that state to CachedGraph's key.
std::vector<Node> build_frame(skb_engine* e, int n_active) {
    const int R = n_active * e->rpr;
    std::vector<Node> nodes;
    // debug timeline: one stamp block per launch of the frame
    auto stamps = [e, &nodes]() { return node_stamps(e, nodes.size()); };
    const std::vector<Phase> phases = build_phases(e, n_active);
    size_t first = 0;
    if (R == 2 && e->dh_ok) {
        // one CFG request on the GEMV path: the 16 depth steps as one
        // persistent cooperative launch (its phases are the first 3 Q)
        DepthArgs da = {};
        da.V = e->V;
        da.Q = e->Q;
        da.rms_eps = e->m.rms_eps;
        da.depth_eps = e->m.depth_eps;
        da.scale = e->m.frame_scale;
        da.final_norm = e->m.final_norm;
        da.norm_in = e->m.depth_norm_in;
        da.norm_out = e->m.depth_norm_out;
        da.wg = e->m.depth_gate;
        da.wu = e->m.depth_up;
        da.wd = e->m.depth_down;
        da.table = e->m.table;
        da.bias = e->m.depth_bias;
        da.x = e->x;
        da.act = e->act;
        da.y = e->y;
        da.hidden = e->hidden;
        da.logits = e->debug ? e->logits_hist : e->logits;
        da.logits_q_stride = e->debug ? e->R * e->V : 0;
        da.st = e->st;
        da.host_flag = e->host_flag;
        da.cur_codes = e->cur_codes;
        da.hist = e->hist;
        da.max_frames = e->o.max_frames;
        da.bos = e->m.bos_id;
        da.pad = e->m.pad_id;
        da.eos = e->m.eos_id;
        da.bar = e->dh_bar;
        da.abort = e->dh_abort;
        da.err = e->err;
        da.ts = e->debug ? e->dh_ts : nullptr;
        const int grid = e->nsm;
        Node n;
        n.w.push_back({(const char*)e->m.depth_gate, (unsigned long long)e->I * e->D * 4});
        n.w.push_back({(const char*)e->m.depth_up, (unsigned long long)e->I * e->D * 4});
        n.ctas = grid;
        n.run = [da, grid](cudaStream_t s, bool, const PrefetchList&) { return depth_head_launch(da, grid, s); };
        nodes.push_back(n);
        first = (size_t)3 * e->Q;
    }
    for (size_t pi = first; pi < phases.size(); ++pi) {
        const Phase& ph = phases[pi];
        if (ph.kind == PH_GEMV) {
            GemvArgs g = ph.g;
            g.ts = stamps();
            if (R >= e->gemm_min_rows)
                gemm_rows_nodes(e, ph, R, nodes);
            else
                nodes.push_back(gemv_node(e, g, R, ph.xm, ph.em));
            if (ph.sample) {
                DepthSampleArgs a = ph.s;
                a.ts = stamps();
                Node n;
                n.ctas = n_active;
                n.run = [a, n_active](cudaStream_t s, bool pdl, const PrefetchList& pf) {
                    DepthSampleArgs b = a;
                    b.pf = pf;
                    if (b.V <= DEPTH_VMAX_SMALL)
                        return launch(depth_sample_kernel<DEPTH_VMAX_SMALL>, dim3(n_active), dim3(SAMPLER_THREADS),
                                      sampler_smem_bytes<DEPTH_VMAX_SMALL>(), s, pdl, b);
                    return launch(depth_sample_kernel<SAMPLER_VMAX>, dim3(n_active), dim3(SAMPLER_THREADS),
                                  sampler_smem_bytes<SAMPLER_VMAX>(), s, pdl, b);
                };
                nodes.push_back(n);
            }
        } else {
            DecodeAttnArgs a = ph.at;
            a.ts = stamps();
            Node n;
            n.ctas = a.S * e->KVH * R;
            n.run = [a, R](cudaStream_t s, bool pdl, const PrefetchList& pf) {
                DecodeAttnArgs b = a;
                b.pf = pf;
                return decode_attn_cluster_launch(b, R, s, pdl);
            };
            nodes.push_back(n);
        }
    }
    e->frame_nodes = (int)nodes.size();
    return nodes;
}

PrefetchList make_pf(const std::vector<WRange>& w, bool on) {
    PrefetchList pf = {};
    if (!on) return pf;
    for (size_t i = 0; i < w.size() && i < 4; ++i) {
        pf.ptr[pf.n] = w[i].p;
        pf.bytes[pf.n] = w[i].bytes;
        ++pf.n;
    }
    return pf;
}

// Prefetch policy: a kernel with at least 64 CTAs prefetches the weights of
// the next kernel that reads weights, looking past one narrow, weightless
// kernel (the sampler).  Narrow kernels never prefetch: one CTA issuing a
// whole weight set is limited by its SM's request rate.
PrefetchList prefetch_for(const skb_engine* e, const std::vector<Node>& nodes, size_t i) {
    const size_t n = nodes.size();
    if (!e->o.l2_prefetch || nodes[i].ctas < 64) return make_pf({}, false);
    const Node& n1 = nodes[(i + 1) % n];
    if (!n1.w.empty()) return make_pf(n1.w, true);
    if (n1.ctas < 64) {
        const Node& n2 = nodes[(i + 2) % n];
        if (!n2.w.empty()) return make_pf(n2.w, true);
    }
    return make_pf({}, false);
}

int run_frames(skb_engine* e, const std::vector<Node>& nodes, int frames, cudaStream_t s, bool pdl) {
    const size_t n = nodes.size();
    for (int f = 0; f < frames; ++f) {
        for (size_t i = 0; i < n; ++i) {
            const PrefetchList pf = prefetch_for(e, nodes, i);
            const bool use_pdl = pdl && !(f == 0 && i == 0);
            cudaError_t err = nodes[i].run(s, use_pdl, pf);
            if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "frame kernel %zu: %s", i, cudaGetErrorString(err));
        }
    }
    return SKB_OK;
}

constexpr size_t GRAPH_CACHE = 16;

// Drops every captured graph (the frame program changed, or the engine goes).
void destroy_graph(skb_engine* e) {
    for (auto& g : e->graphs) cudaGraphExecDestroy(g.exec);
    e->graphs.clear();
    e->exec = nullptr;
    e->graph_active = 0;
    e->graph_fpg = 0;
}

int upload_state(skb_engine* e, int req, cudaStream_t s) {
    cudaError_t err = cudaMemcpyAsync(e->st + req, &e->st_host[req], sizeof(ReqState),
                                      cudaMemcpyHostToDevice, s);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "state upload: %s", cudaGetErrorString(err));
    return SKB_OK;
}

}  // namespace

extern "C" {

int skb_engine_create(const skb_model_desc* md, const skb_engine_opts* opts, skb_engine** out) {
    if (!md || !opts || !out) return fail(SKB_ERR_ARG, "engine_create: null argument");
    *out = nullptr;
    const skb_model_desc& m = *md;
    if (m.head_dim != 128) return fail(SKB_ERR_ARG, "head_dim must be 128 (got %d)", m.head_dim);
    if (m.n_heads % m.n_kv_heads != 0 || m.n_heads / m.n_kv_heads > 2)
        return fail(SKB_ERR_ARG, "GQA group size must be 1 or 2 (heads %d / kv heads %d)", m.n_heads, m.n_kv_heads);
    // every GEMV inner size must fit the ring GEMV (K <= 3072: a SwiGLU row
    // pair fills one 24 KB slot)
    if (m.d_model % 16 || m.d_model > 3072 || m.ffn_dim % 16 || m.ffn_dim > 3072 || m.depth_inner % 16 ||
        m.depth_inner > 3072 || m.n_heads * m.head_dim > 3072)
        return fail(SKB_ERR_ARG, "model widths must be multiples of 16 and <= 3072");
    if (m.audio_vocab > SAMPLER_VMAX) return fail(SKB_ERR_ARG, "audio vocab %d > %d", m.audio_vocab, SAMPLER_VMAX);
    if (m.n_codebooks > 32 || m.n_codebooks < 1) return fail(SKB_ERR_ARG, "1..32 codebooks supported");
    if (opts->rows_per_request != 1 && opts->rows_per_request != 2)
        return fail(SKB_ERR_ARG, "rows_per_request must be 1 or 2");
    if (opts->max_requests < 1 || opts->max_requests * opts->rows_per_request > 512)
        return fail(SKB_ERR_ARG, "max_requests * rows_per_request must be 1..512");
    if (opts->max_len < 2 || opts->max_frames < 1 || opts->max_prefill < 1 || opts->max_prefill > opts->max_len)
        return fail(SKB_ERR_ARG, "bad capacities (max_len %d, max_frames %d, max_prefill %d)", opts->max_len,
                    opts->max_frames, opts->max_prefill);
    if (!m.rope_inv_freq || !m.layers || !m.embed_tokens || !m.table || !m.depth_bias || !m.final_norm)
        return fail(SKB_ERR_ARG, "engine_create: missing weight pointers");
    for (int i = 0; i < m.n_layers * SKB_LAYER_PTRS; ++i)
        if (!m.layers[i] || !aligned16(m.layers[i])) return fail(SKB_ERR_ARG, "layer weight %d null or unaligned", i);
    {
        const void* need[] = {m.embed_tokens, m.final_norm, m.table, m.depth_bias, m.depth_norm_in,
                              m.depth_norm_out, m.depth_gate, m.depth_up, m.depth_down};
        for (const void* p : need)
            if (!p || !aligned16(p)) return fail(SKB_ERR_ARG, "engine weights must be non-null and 16-byte aligned");
        const void* opt[] = {m.lang_embed, m.speaker_proj, m.speaker_slot};
        for (const void* p : opt)
            if (p && !aligned16(p)) return fail(SKB_ERR_ARG, "engine weights must be 16-byte aligned");
    }

    skb_engine* e = new skb_engine();
    e->m = m;
    e->lw.assign(m.layers, m.layers + (size_t)m.n_layers * SKB_LAYER_PTRS);
    e->m.layers = nullptr;
    e->o = *opts;
    cudaGetDevice(&e->device);
    cudaDeviceGetAttribute(&e->nsm, cudaDevAttrMultiProcessorCount, e->device);
    e->rpr = opts->rows_per_request;
    e->nreq = opts->max_requests;
    e->R = e->nreq * e->rpr;
    e->D = m.d_model;
    e->H = m.n_heads;
    e->KVH = m.n_kv_heads;
    e->hd = m.head_dim;
    e->F = m.ffn_dim;
    e->I = m.depth_inner;
    e->Q = m.n_codebooks;
    e->V = m.audio_vocab;
    e->L = m.n_layers;
    e->n_rep = m.n_heads / m.n_kv_heads;
    int ps = opts->page_size > 0 ? opts->page_size : 64;
    e->page_log2 = 0;
    while ((1 << e->page_log2) < ps) ++e->page_log2;
    e->o.page_size = 1 << e->page_log2;
    e->max_pages = (opts->max_len + e->o.page_size - 1) / e->o.page_size;
    // CTAs per (row, kv head): one cluster, as wide as lets every (row, kv
    // head) cluster be resident at once
    e->S = opts->attn_splits > 0 ? opts->attn_splits : decode_attn_cluster_width(e->R * e->KVH);
    if (e->S > 8) e->S = 8;
    // attention variant by the engine's capacity (the same for every batch width)
    e->attn_variant = e->R * e->KVH > 32 ? 2 : 1;
    e->gemm_min_rows = opts->gemm_min_rows > 0 ? opts->gemm_min_rows : 5;
    e->shared_pool = opts->kv_pages > 0;
    e->pool_pages = e->shared_pool ? opts->kv_pages : e->R * e->max_pages;
    const size_t n_pages = (size_t)e->pool_pages;
    e->layer_floats = (long long)n_pages * 2 * e->KVH * e->o.page_size * e->hd;
    const int qkvd = (e->H + 2 * e->KVH) * e->hd;
    const int actd = e->F > e->I ? e->F : e->I;
    e->prefill_batch = opts->prefill_batch > 0 ? opts->prefill_batch : 1;
    if (e->prefill_batch > e->nreq) e->prefill_batch = e->nreq;
    const int T = e->prefill_batch * e->rpr * opts->max_prefill;
    int st = SKB_OK;
#define A(ptr, n)                          \
    if (st == SKB_OK) st = dalloc(e, &ptr, (size_t)(n));
    A(e->x, (size_t)e->R * e->D)
    A(e->qkv, (size_t)e->R * qkvd)
    A(e->attn, (size_t)e->R * e->H * e->hd)
    A(e->act, (size_t)e->R * actd)
    A(e->abuf, (size_t)e->R * e->D)
    A(e->y, (size_t)e->R * e->D)
    A(e->hidden, (size_t)e->R * e->D)
    A(e->logits, (size_t)e->R * e->V)
    A(e->logits_hist, (size_t)e->Q * e->R * e->V)
    A(e->prefix, (size_t)e->nreq * e->D)
    A(e->rope_cos, (size_t)opts->max_len * (e->hd / 2))
    A(e->rope_sin, (size_t)opts->max_len * (e->hd / 2))
    A(e->kv, (size_t)e->L * e->layer_floats)
    A(e->pos, e->R)
    A(e->page_table, (size_t)e->R * e->max_pages)
    A(e->err, 8)
    A(e->kts, (size_t)SKB_KTS_STRIDE * kts_slots(e))
    if (e->R >= e->gemm_min_rows) A(e->xn, (size_t)e->R * 3072)
    A(e->pt_tmp, (size_t)e->max_pages)
    A(e->host_flag, 1)
    A(e->cur_codes, (size_t)e->nreq * e->Q)
    A(e->hist, (size_t)e->nreq * opts->max_frames * e->Q)
    A(e->st, e->nreq)
    A(e->pX, (size_t)T * e->D)
    A(e->pN, (size_t)T * e->D)
    A(e->pQKV, (size_t)T * qkvd)
    A(e->pQ, (size_t)T * e->H * e->hd)
    A(e->pA, (size_t)T * e->H * e->hd)
    A(e->pG, (size_t)T * e->F)
    A(e->spk, e->D)
    A(e->spk_in, m.speaker_dim > 0 ? m.speaker_dim : 1)
    A(e->ptok, T)
    A(e->pframes, (size_t)e->prefill_batch * (opts->max_prefill + 1) * e->Q)
    A(e->pmeta, (size_t)5 * e->prefill_batch * e->rpr)
    A(e->dh_bar, 1)
    A(e->dh_abort, 1)
    A(e->dh_ts, (size_t)2 * depth_head_phases(e->Q))
#undef A
    if (st != SKB_OK) {
        skb_engine_destroy(e);
        return st;
    }
    // RoPE tables: cos/sin of the fp32 angle inv_freq[i] * p (modeling_qwen3.py:130-146)
    {
        const int half = e->hd / 2;
        std::vector<float> c((size_t)opts->max_len * half), s((size_t)opts->max_len * half);
        for (int p = 0; p < opts->max_len; ++p)
            for (int i = 0; i < half; ++i) {
                const float ang = (float)p * m.rope_inv_freq[i];
                c[(size_t)p * half + i] = (float)std::cos((double)ang);
                s[(size_t)p * half + i] = (float)std::sin((double)ang);
            }
        cudaMemcpy(e->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(e->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice);
    }
    {  // own pages: row r holds [r*max_pages, (r+1)*max_pages); shared pool: unmapped
        e->pt_host.assign((size_t)e->R * e->max_pages, -1);
        if (!e->shared_pool)
            for (size_t i = 0; i < e->pt_host.size(); ++i) e->pt_host[i] = (int)i;
        cudaMemcpy(e->page_table, e->pt_host.data(), e->pt_host.size() * 4, cudaMemcpyHostToDevice);
    }
    e->frames_host.assign(e->nreq, 0);
    e->pos_host.assign(e->R, 0);
    e->st_host.assign(e->nreq, ReqState{});
    for (int r = 0; r < e->nreq; ++r) {
        ReqState& s = e->st_host[r];
        s.stream = (unsigned)r;
        s.cfg = 1.5f;
        s.temp = s.temp_q0 = 0.9f;
        s.top_k = s.top_k_q0 = 50;
        s.top_p = s.top_p_q0 = 0.95f;
        s.min_new_frames = 0;
        s.eos_rule = 0;
    }
    cudaMemcpy(e->st, e->st_host.data(), sizeof(ReqState) * e->nreq, cudaMemcpyHostToDevice);
    e->dh_ok = e->rpr == 2 && !opts->split_depth_head && e->gemm_min_rows > 2 &&
               depth_head_supported(e->D, e->I, e->V, e->Q, e->nsm, e->device);
    if (cudaHostAlloc(reinterpret_cast<void**>(&e->err_host), 8 * sizeof(int), cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->err_ev, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        skb_engine_destroy(e);
        return fail(SKB_ERR_CUDA, "engine_create: error-flag mirror");
    }
    memset(e->err_host, 0, 8 * sizeof(int));
    if (cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
        skb_engine_destroy(e);
        return fail(SKB_ERR_CUDA, "stream creation failed");
    }
    set_smem_attrs(depth_sample_kernel<DEPTH_VMAX_SMALL>, sampler_smem_bytes<DEPTH_VMAX_SMALL>());
    set_smem_attrs(depth_sample_kernel<SAMPLER_VMAX>, sampler_smem_bytes<SAMPLER_VMAX>());
    decode_attn_cluster_prepare();
    depth_head_prepare();
    trunk_init_attrs();
    gemv_prepare_all();
    tgemm_prepare();
    const cudaError_t ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) {
        skb_engine_destroy(e);
        return fail(SKB_ERR_CUDA, "engine init: %s", cudaGetErrorString(ce));
    }
    *out = e;
    return SKB_OK;
}

int skb_engine_destroy(skb_engine* e) {
    if (!e) return SKB_OK;
    destroy_graph(e);
    if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
    if (e->err_ev) cudaEventDestroy(e->err_ev);
    if (e->err_host) cudaFreeHost(e->err_host);
    for (void* p : e->allocs) cudaFree(p);
    delete e;
    return SKB_OK;
}

// Shared pool: the row's positions [0, n) must sit on mapped pages.
static int check_pages(const skb_engine* e, int row, int n) {
    if (!e->shared_pool) return SKB_OK;
    const int need = (n + e->o.page_size - 1) >> e->page_log2;
    for (int p = 0; p < need && p < e->max_pages; ++p)
        if (e->pt_host[(size_t)row * e->max_pages + p] < 0)
            return fail(SKB_ERR_CAPACITY, "row %d: KV page %d (positions %d..) is not mapped", row, p,
                        p * e->o.page_size);
    return SKB_OK;
}

int skb_engine_set_sampling(skb_engine* e, int req, float cfg, float temp, float temp_q0, int top_k,
                            float top_p, int top_k_q0, float top_p_q0, uint64_t seed, int min_new_frames,
                            int eos_rule) {
    if (!e || req < 0 || req >= e->nreq) return fail(SKB_ERR_ARG, "set_sampling: bad request %d", req);
    ReqState& s = e->st_host[req];
    s.cfg = cfg;
    s.temp = temp;
    s.temp_q0 = temp_q0;
    s.top_k = (top_k > 0 && top_k < e->V) ? top_k : 0;
    s.top_k_q0 = (top_k_q0 > 0 && top_k_q0 < e->V) ? top_k_q0 : 0;
    s.top_p = (top_p > 0.f && top_p < 1.f) ? top_p : -1.f;
    s.top_p_q0 = (top_p_q0 > 0.f && top_p_q0 < 1.f) ? top_p_q0 : -1.f;
    s.seed = seed;
    s.min_new_frames = min_new_frames;
    s.eos_rule = eos_rule;
    // frame / done counters live on the device; upload only the parameters
    const size_t n = offsetof(ReqState, frame);
    cudaError_t err1 = cudaMemcpy(e->st + req, &s, n, cudaMemcpyHostToDevice);
    cudaError_t err2 = cudaMemcpy(reinterpret_cast<char*>(e->st + req) + offsetof(ReqState, seed), &s.seed,
                                  sizeof(s.seed), cudaMemcpyHostToDevice);
    if (err1 != cudaSuccess || err2 != cudaSuccess) return fail(SKB_ERR_CUDA, "set_sampling upload failed");
    return SKB_OK;
}

// The prompts of n requests (reqs[i]'s cond / uncond ids, reference frames
// and, for n == 1 only, speaker vector) through the trunk in one pass: their
// tokens are concatenated (rows keep their own positions), so every GEMM of
// the pass sees all of them.
static int prefill_impl(skb_engine* e, int n, const int* reqs, const int64_t* const* conds, const int* n_conds,
                        const int64_t* const* unconds, const int* n_unconds, const int64_t* const* prompts,
                        const int* n_prompts, const float* speaker, cudaStream_t s) {
    if (n < 1 || n > e->prefill_batch)
        return fail(SKB_ERR_ARG, "prefill: %d requests (1..%d per pass, opts.prefill_batch)", n, e->prefill_batch);
    const skb_model_desc& m = e->m;
    const bool use_spk = speaker != nullptr;
    if (use_spk && !m.speaker_proj) return fail(SKB_ERR_ARG, "speaker embedding supplied to an unconditioned model");
    if (!use_spk && m.speaker_proj) return fail(SKB_ERR_ARG, "this model requires a speaker embedding");
    if (use_spk && n != 1) return fail(SKB_ERR_ARG, "prefill: speaker vectors go one request per pass");
    const bool slot = use_spk && m.speaker_slot_mode;
    if (slot && !m.speaker_slot) return fail(SKB_ERR_ARG, "slot mode without speaker_slot_embedding");
    auto is_lang = [&](int64_t id) {
        for (int j = 0; j < m.n_lang; ++j)
            if (m.lang_ids[j] == id) return true;
        return false;
    };
    for (int i = 0; i < n; ++i) {
        const int req = reqs[i];
        if (req < 0 || req >= e->nreq) return fail(SKB_ERR_ARG, "prefill: bad request %d", req);
        for (int j = 0; j < i; ++j)
            if (reqs[j] == req) return fail(SKB_ERR_ARG, "prefill: request %d given twice", req);
        if (!conds[i] || n_conds[i] < 1) return fail(SKB_ERR_ARG, "prefill: empty cond ids");
        if (e->rpr == 2 && (!unconds[i] || n_unconds[i] < 1)) return fail(SKB_ERR_ARG, "prefill: CFG needs uncond ids");
        if (n_prompts[i] < 0 || (n_prompts[i] > 0 && !prompts[i])) return fail(SKB_ERR_ARG, "prefill: bad prompt codes");
        for (int b = 0; b < e->rpr; ++b) {
            const int64_t* ids = b == 0 ? conds[i] : unconds[i];
            const int nn = b == 0 ? n_conds[i] : n_unconds[i];
            for (int k = 0; k < nn; ++k)
                if ((ids[k] < 0 || ids[k] >= m.text_vocab) && !is_lang(ids[k]))
                    return fail(SKB_ERR_ARG, "prefill: text id %lld out of range", (long long)ids[k]);
        }
        for (int k = 0; k < n_prompts[i] * e->Q; ++k)
            if (prompts[i][k] < 0 || prompts[i][k] >= e->V) return fail(SKB_ERR_ARG, "prefill: prompt code out of range");
    }
    // tokens of every row; each request's frames (audio BOS + prompt) in one array
    const int NR = n * e->rpr;
    std::vector<PrefillTok> toks;
    std::vector<int> row_off(NR), row_len(NR), row_id(NR);
    std::vector<int64_t> frames;
    for (int i = 0; i < n; ++i) {
        const int fbase = (int)(frames.size() / e->Q);
        for (int q = 0; q < e->Q; ++q) frames.push_back(m.bos_id);
        frames.insert(frames.end(), prompts[i], prompts[i] + (size_t)n_prompts[i] * e->Q);
        for (int b = 0; b < e->rpr; ++b) {
            const int k = i * e->rpr + b;
            const int row = reqs[i] * e->rpr + b;
            const int64_t* ids = b == 0 ? conds[i] : unconds[i];
            const int nn = b == 0 ? n_conds[i] : n_unconds[i];
            row_off[k] = (int)toks.size();
            int p = 0;
            for (int t = 0; t < nn; ++t) toks.push_back({row, p++, 0, (int)ids[t]});
            if (slot) toks.push_back({row, p++, 2, 0});
            for (int f = 0; f <= n_prompts[i]; ++f) toks.push_back({row, p++, 1, fbase + f});
            row_len[k] = p;
            row_id[k] = row;
            if (p > e->o.max_prefill || p >= e->o.max_len)
                return fail(SKB_ERR_CAPACITY, "prefill %d exceeds max_prefill=%d / max_len=%d", p, e->o.max_prefill,
                            e->o.max_len);
            const int pst = check_pages(e, row, p);
            if (pst) return pst;
        }
    }
    const int T = (int)toks.size();
    const int RC = e->prefill_batch * e->rpr;  // pmeta stride
    std::vector<int> meta((size_t)5 * RC, 0);
    int maxL = 0;
    for (int k = 0; k < NR; ++k) {
        meta[0 * RC + k] = row_off[k];
        meta[1 * RC + k] = row_len[k];
        meta[2 * RC + k] = row_id[k];
        meta[3 * RC + k] = row_off[k] + row_len[k] - 1;
        meta[4 * RC + k] = row_id[k];
        maxL = row_len[k] > maxL ? row_len[k] : maxL;
    }
    cudaError_t err = cudaSuccess;
#define CK(x)                                                                        \
    do {                                                                             \
        err = (x);                                                                   \
        if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "prefill %s: %s", #x, cudaGetErrorString(err)); \
    } while (0)
    CK(cudaMemcpyAsync(e->ptok, toks.data(), sizeof(PrefillTok) * T, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(e->pframes, frames.data(), frames.size() * 8, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(e->pmeta, meta.data(), sizeof(int) * meta.size(), cudaMemcpyHostToDevice, s));
    const float* bos_add = nullptr;
    if (use_spk) {
        CK(cudaMemcpyAsync(e->spk_in, speaker, sizeof(float) * m.speaker_dim, cudaMemcpyHostToDevice, s));
        CK(speaker_launch(e->spk_in, m.speaker_dim, m.speaker_proj, e->D, slot ? m.speaker_slot : nullptr, e->spk, s));
        if (!slot) bos_add = e->spk;  // (one request: its audio BOS frame is frame 0)
    }
    CK(prefill_embed_launch(e->ptok, T, m.embed_tokens, m.text_vocab, m.lang_embed, m.n_lang, m.lang_ids,
                            e->pframes, e->Q, m.table, e->V, m.frame_scale, e->spk, bos_add, e->pX, e->D,
                            e->err + 1, s));
    const KVLayout kv = kv_layout(e);
    const int qd = e->H * e->hd, kvd = e->KVH * e->hd;
    for (int l = 0; l < e->L; ++l) {
        int stt = rmsnorm_rows(e->pX, nullptr, LW(e, l, W_LN1), e->pN, T, e->D, m.rms_eps, s, false);
        if (stt) return stt;
        GemmArgs g = {};
        g.A = e->pN;
        g.lda = e->D;
        g.w0 = LW(e, l, W_Q);
        g.w1 = LW(e, l, W_K);
        g.w2 = LW(e, l, W_V);
        g.seg1 = qd;
        g.seg2 = qd + kvd;
        g.N = qd + 2 * kvd;
        g.K = e->D;
        g.T = T;
        g.out = e->pQKV;
        g.ldo = qd + 2 * kvd;
        g.mode = 0;
        CK(tgemm_launch(g, s));
        CK(prefill_qk_launch(e->pQKV, qd + 2 * kvd, e->ptok, T, LW(e, l, W_QN), LW(e, l, W_KN), m.rms_eps,
                             e->rope_cos, e->rope_sin, e->H, kv, l, e->pQ, s));
        CK(prefill_attn_launch(e->pQ, e->pmeta, e->pmeta + RC, e->pmeta + 2 * RC, NR, maxL, e->H, e->n_rep, kv, l,
                               1.0f / sqrtf((float)e->hd), e->pA, s));
        GemmArgs o = {};
        o.A = e->pA;
        o.lda = qd;
        o.w0 = LW(e, l, W_O);
        o.seg1 = o.seg2 = 1 << 30;
        o.N = e->D;
        o.K = qd;
        o.T = T;
        o.out = e->pX;
        o.ldo = e->D;
        o.resid = e->pX;
        o.ldr = e->D;
        o.mode = 1;
        CK(tgemm_launch(o, s));
        stt = rmsnorm_rows(e->pX, nullptr, LW(e, l, W_LN2), e->pN, T, e->D, m.rms_eps, s, false);
        if (stt) return stt;
        GemmArgs gu = {};
        gu.A = e->pN;
        gu.lda = e->D;
        gu.w0 = LW(e, l, W_G);
        gu.w1 = LW(e, l, W_U);
        gu.interleave = 1;
        gu.N = 2 * e->F;
        gu.K = e->D;
        gu.T = T;
        gu.out = e->pG;
        gu.ldo = e->F;
        gu.mode = 3;
        CK(tgemm_launch(gu, s));
        GemmArgs dn = {};
        dn.A = e->pG;
        dn.lda = e->F;
        dn.w0 = LW(e, l, W_D);
        dn.seg1 = dn.seg2 = 1 << 30;
        dn.N = e->D;
        dn.K = e->F;
        dn.T = T;
        dn.out = e->pX;
        dn.ldo = e->D;
        dn.resid = e->pX;
        dn.ldr = e->D;
        dn.mode = 1;
        CK(tgemm_launch(dn, s));
    }
    CK(gather_rows_launch(e->pX, e->pmeta + 3 * RC, e->pmeta + 4 * RC, NR, e->x, e->D, s));
    // positions, prefix, counters of each request
    for (int i = 0; i < n; ++i) {
        const int req = reqs[i];
        CK(cudaMemcpyAsync(e->pos + req * e->rpr, row_len.data() + i * e->rpr, sizeof(int) * e->rpr,
                           cudaMemcpyHostToDevice, s));
        CK(cudaMemsetAsync(e->prefix + (size_t)req * e->D, 0, sizeof(float) * e->D, s));
        static const int zero2[2] = {0, 0};
        CK(cudaMemcpyAsync(reinterpret_cast<char*>(e->st + req) + offsetof(ReqState, frame), zero2, sizeof zero2,
                           cudaMemcpyHostToDevice, s));
    }
    CK(cudaStreamSynchronize(s));
#undef CK
    for (int i = 0; i < n; ++i) {
        for (int b = 0; b < e->rpr; ++b) e->pos_host[reqs[i] * e->rpr + b] = row_len[i * e->rpr + b];
        e->frames_host[reqs[i]] = 0;
    }
    return SKB_OK;
}

int skb_engine_prefill(skb_engine* e, int req, const int64_t* cond, int n_cond, const int64_t* uncond,
                       int n_uncond, const int64_t* prompt, int n_prompt, const float* speaker,
                       cudaStream_t s) {
    if (!e) return fail(SKB_ERR_ARG, "prefill: null engine");
    return prefill_impl(e, 1, &req, &cond, &n_cond, &uncond, &n_uncond, &prompt, &n_prompt, speaker, s);
}

int skb_engine_prefill_many(skb_engine* e, int n, const int* requests, const int64_t* const* cond_ids,
                            const int* n_cond, const int64_t* const* uncond_ids, const int* n_uncond,
                            const int64_t* const* prompt_codes, const int* n_prompt, cudaStream_t s) {
    if (!e || n < 1 || !requests || !cond_ids || !n_cond || !n_prompt || (e->rpr == 2 && (!uncond_ids || !n_uncond)))
        return fail(SKB_ERR_ARG, "prefill_many: bad arguments");
    std::vector<const int64_t*> unc(n, nullptr), pc(n, nullptr);
    std::vector<int> nu(n, 0);
    for (int i = 0; i < n; ++i) {
        if (uncond_ids) unc[i] = uncond_ids[i];
        if (n_uncond) nu[i] = n_uncond[i];
        if (prompt_codes) pc[i] = prompt_codes[i];
    }
    return prefill_impl(e, n, requests, cond_ids, n_cond, unc.data(), nu.data(), pc.data(), n_prompt, nullptr, s);
}

int skb_engine_capture(skb_engine* e, int n_active, int fpg, cudaStream_t stream) {
    if (!e) return fail(SKB_ERR_ARG, "capture: null engine");
    if (n_active < 1 || n_active > e->nreq || fpg < 1 || fpg > 64)
        return fail(SKB_ERR_ARG, "capture: n_active %d (1..%d), frames_per_graph %d (1..64)", n_active, e->nreq, fpg);
    for (auto& g : e->graphs)
        if (g.n_active == n_active && g.fpg == fpg) {  // captured before: reuse it
            g.used = ++e->graph_clock;
            e->exec = g.exec;
            e->graph_active = n_active;
            e->graph_fpg = fpg;
            e->graph_pdl = g.pdl;
            return SKB_OK;
        }
    if (e->graphs.size() >= GRAPH_CACHE) {
        size_t lru = 0;
        for (size_t i = 1; i < e->graphs.size(); ++i)
            if (e->graphs[i].used < e->graphs[lru].used) lru = i;
        if (e->graphs[lru].exec == e->exec) e->exec = nullptr;
        cudaGraphExecDestroy(e->graphs[lru].exec);
        e->graphs.erase(e->graphs.begin() + (long)lru);
    }
    cudaStream_t cs = e->cap_stream;
    cudaError_t err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "capture sync: %s", cudaGetErrorString(err));
    const std::vector<Node> nodes = build_frame(e, n_active);
    for (int attempt = 0; attempt < 2; ++attempt) {
        const bool pdl = e->o.use_pdl && attempt == 0;
        cudaGraph_t graph = nullptr;
        err = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "begin capture: %s", cudaGetErrorString(err));
        int st = run_frames(e, nodes, fpg, cs, pdl);
        err = cudaStreamEndCapture(cs, &graph);
        if (st != SKB_OK || err != cudaSuccess) {
            cudaGetLastError();
            if (graph) cudaGraphDestroy(graph);
            if (pdl) continue;
            return st != SKB_OK ? st : fail(SKB_ERR_CUDA, "end capture: %s", cudaGetErrorString(err));
        }
        err = cudaGraphInstantiate(&e->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (err != cudaSuccess) {
            cudaGetLastError();
            e->exec = nullptr;
            if (pdl) continue;
            return fail(SKB_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(err));
        }
        e->graph_active = n_active;
        e->graph_fpg = fpg;
        e->graph_pdl = pdl ? 1 : 0;
        e->graphs.push_back({n_active, fpg, e->graph_pdl, e->exec, ++e->graph_clock});
        return SKB_OK;
    }
    return fail(SKB_ERR_CUDA, "capture failed");
}

static int check_capacity(skb_engine* e, int n_active, int frames) {
    for (int r = 0; r < n_active; ++r) {
        for (int b = 0; b < e->rpr; ++b) {
            const int row = r * e->rpr + b;
            const int st = check_pages(e, row, e->pos_host[row] + frames);
            if (st) return st;
        }
        if (e->frames_host[r] + frames > e->o.max_frames)
            return fail(SKB_ERR_CAPACITY, "frame buffer full (%d + %d > max_frames %d)", e->frames_host[r], frames,
                        e->o.max_frames);
        for (int b = 0; b < e->rpr; ++b)
            if (e->pos_host[r * e->rpr + b] + frames > e->o.max_len)
                return fail(SKB_ERR_CAPACITY, "KV cache full (position %d + %d > max_len %d)",
                            e->pos_host[r * e->rpr + b], frames, e->o.max_len);
    }
    return SKB_OK;
}

static void advance_host(skb_engine* e, int n_active, int frames) {
    for (int r = 0; r < n_active; ++r) {
        e->frames_host[r] += frames;
        for (int b = 0; b < e->rpr; ++b) e->pos_host[r * e->rpr + b] += frames;
    }
}

// Device error flags: 0 a position out of range (attention), 1 a prefill
// token id or code out of range, 2 a weight copy that did not arrive in time
// (GEMV / tensor-core GEMM).  Once a flag has been observed every later step
// fails: the engine's state can no longer be trusted.
static const char* const kFlagWhat[8] = {"position out of range", "prefill input out of range",
                                         "a weight copy did not arrive in time", "flag 3", "flag 4", "flag 5",
                                         "flag 6", "flag 7"};
static int flag_status(skb_engine* e) {
    if (e->err_seen < 0) {
        for (int i = 0; i < 8; ++i)
            if (e->err_host[i] != 0) {
                e->err_seen = i;
                break;
            }
    }
    if (e->err_seen >= 0)
        return fail(SKB_ERR_CUDA, "device error flag %d raised by an earlier launch (%s)", e->err_seen,
                    kFlagWhat[e->err_seen]);
    return SKB_OK;
}

// Checks the flags copied by an earlier step, without waiting for the copy.
static int check_flags_async(skb_engine* e) {
    if (e->err_pending && cudaEventQuery(e->err_ev) == cudaSuccess) e->err_pending = false;
    if (e->err_pending) return e->err_seen >= 0 ? flag_status(e) : SKB_OK;
    return flag_status(e);
}

// Queues a copy of the device flags behind the work already on `stream`.
static void queue_flag_copy(skb_engine* e, cudaStream_t stream) {
    if (e->err_pending) return;
    if (cudaMemcpyAsync(e->err_host, e->err, 8 * sizeof(int), cudaMemcpyDeviceToHost, stream) == cudaSuccess &&
        cudaEventRecord(e->err_ev, stream) == cudaSuccess)
        e->err_pending = true;
    else
        cudaGetLastError();
}

int skb_engine_step(skb_engine* e, int mask_eos_q0, cudaStream_t stream) {
    if (!e) return fail(SKB_ERR_ARG, "step: null engine");
    if (!e->exec) return fail(SKB_ERR_STATE, "call capture() first");
    int st = check_flags_async(e);
    if (st) return st;
    st = check_capacity(e, e->graph_active, e->graph_fpg);
    if (st) return st;
    static thread_local int flag_val;
    flag_val = mask_eos_q0 ? 1 : 0;
    cudaError_t err = cudaMemcpyAsync(e->host_flag, &flag_val, sizeof(int), cudaMemcpyHostToDevice, stream);
    if (err == cudaSuccess) err = cudaGraphLaunch(e->exec, stream);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "step: %s", cudaGetErrorString(err));
    queue_flag_copy(e, stream);
    advance_host(e, e->graph_active, e->graph_fpg);
    return SKB_OK;
}

int skb_engine_step_eager(skb_engine* e, int n_active, int mask_eos_q0, cudaStream_t stream) {
    if (!e || n_active < 1 || n_active > e->nreq) return fail(SKB_ERR_ARG, "step_eager: bad arguments");
    int st = check_capacity(e, n_active, 1);
    if (st) return st;
    static thread_local int flag_val;
    flag_val = mask_eos_q0 ? 1 : 0;
    cudaError_t err = cudaMemcpyAsync(e->host_flag, &flag_val, sizeof(int), cudaMemcpyHostToDevice, stream);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "step_eager: %s", cudaGetErrorString(err));
    const std::vector<Node> nodes = build_frame(e, n_active);
    st = run_frames(e, nodes, 1, stream, false);
    if (st) return st;
    advance_host(e, n_active, 1);
    return SKB_OK;
}

int skb_engine_read_codes(skb_engine* e, int req, int first, int n, int64_t* dst, cudaStream_t stream) {
    if (!e || req < 0 || req >= e->nreq || first < 0 || n < 0 || first + n > e->o.max_frames || (n > 0 && !dst))
        return fail(SKB_ERR_ARG, "read_codes: bad arguments");
    if (n == 0) return SKB_OK;
    cudaError_t err = cudaMemcpyAsync(dst, e->hist + ((size_t)req * e->o.max_frames + first) * e->Q,
                                      sizeof(int64_t) * n * e->Q, cudaMemcpyDefault, stream);
    return err == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "read_codes: %s", cudaGetErrorString(err));
}

int skb_engine_frames(skb_engine* e, int req) {
    if (!e || req < 0 || req >= e->nreq) return -1;
    return e->frames_host[req];
}

int skb_engine_map_pages(skb_engine* e, int row, int first, int n, const int32_t* pages) {
    if (!e || row < 0 || row >= e->R || first < 0 || n < 0 || first + n > e->max_pages || (n > 0 && !pages))
        return fail(SKB_ERR_ARG, "map_pages: bad arguments (row %d, pages [%d, %d))", row, first, first + n);
    if (!e->shared_pool) return fail(SKB_ERR_STATE, "map_pages: the engine was created without a shared KV pool");
    for (int i = 0; i < n; ++i)
        if (pages[i] < -1 || pages[i] >= e->pool_pages)
            return fail(SKB_ERR_ARG, "map_pages: page %d outside the pool of %d", pages[i], e->pool_pages);
    if (n == 0) return SKB_OK;
    const cudaError_t err = cudaMemcpy(e->page_table + (size_t)row * e->max_pages + first, pages, sizeof(int) * n,
                                       cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "map_pages: %s", cudaGetErrorString(err));
    for (int i = 0; i < n; ++i) e->pt_host[(size_t)row * e->max_pages + first + i] = pages[i];
    return SKB_OK;
}

int skb_engine_set_rng_stream(skb_engine* e, int req, uint32_t stream) {
    if (!e || req < 0 || req >= e->nreq) return fail(SKB_ERR_ARG, "set_rng_stream: bad request %d", req);
    e->st_host[req].stream = stream;
    const cudaError_t err = cudaMemcpy(reinterpret_cast<char*>(e->st + req) + offsetof(ReqState, stream), &stream,
                                       sizeof(stream), cudaMemcpyHostToDevice);
    return err == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "set_rng_stream: %s", cudaGetErrorString(err));
}

int skb_engine_status(skb_engine* e, int n, int32_t* frames, int32_t* done, cudaStream_t s) {
    if (!e || n < 0 || n > e->nreq || (n > 0 && (!frames || !done)))
        return fail(SKB_ERR_ARG, "status: bad arguments");
    if (n == 0) return SKB_OK;
    std::vector<ReqState> tmp(n);
    cudaError_t err = cudaMemcpyAsync(tmp.data(), e->st, sizeof(ReqState) * n, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess && e->err_pending) err = cudaEventSynchronize(e->err_ev);
    e->err_pending = false;
    if (err == cudaSuccess) err = cudaMemcpy(e->err_host, e->err, 8 * sizeof(int), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "status: %s", cudaGetErrorString(err));
    const int fst = flag_status(e);
    if (fst) return fst;
    for (int r = 0; r < n; ++r) {
        frames[r] = tmp[r].frame;
        done[r] = tmp[r].done;
    }
    return SKB_OK;
}

int skb_engine_move_request(skb_engine* e, int dst, int src, cudaStream_t s) {
    if (!e || dst < 0 || dst >= e->nreq || src < 0 || src >= e->nreq)
        return fail(SKB_ERR_ARG, "move_request: bad slots %d <- %d", dst, src);
    if (dst == src) return SKB_OK;
    const size_t D = (size_t)e->D, Q = (size_t)e->Q, MF = (size_t)e->o.max_frames, MP = (size_t)e->max_pages;
    cudaError_t err = cudaSuccess;
    auto cp = [&](void* d, const void* sp, size_t bytes) {
        if (err == cudaSuccess) err = cudaMemcpyAsync(d, sp, bytes, cudaMemcpyDeviceToDevice, s);
    };
    cp(e->st + dst, e->st + src, sizeof(ReqState));
    cp(e->cur_codes + dst * Q, e->cur_codes + src * Q, sizeof(int64_t) * Q);
    cp(e->hist + dst * MF * Q, e->hist + src * MF * Q, sizeof(int64_t) * MF * Q);
    cp(e->prefix + dst * D, e->prefix + src * D, sizeof(float) * D);
    for (int b = 0; b < e->rpr; ++b) {
        const size_t rd = (size_t)dst * e->rpr + b, rs = (size_t)src * e->rpr + b;
        cp(e->x + rd * D, e->x + rs * D, sizeof(float) * D);
        cp(e->pos + rd, e->pos + rs, sizeof(int));
        // exchange page-table rows: the pages stay unique, the KV stays put
        cp(e->pt_tmp, e->page_table + rd * MP, sizeof(int) * MP);
        cp(e->page_table + rd * MP, e->page_table + rs * MP, sizeof(int) * MP);
        cp(e->page_table + rs * MP, e->pt_tmp, sizeof(int) * MP);
        for (size_t p = 0; p < MP; ++p) std::swap(e->pt_host[rd * MP + p], e->pt_host[rs * MP + p]);
        e->pos_host[rd] = e->pos_host[rs];
    }
    if (err != cudaSuccess) return fail(SKB_ERR_CUDA, "move_request: %s", cudaGetErrorString(err));
    e->st_host[dst] = e->st_host[src];
    e->frames_host[dst] = e->frames_host[src];
    return SKB_OK;
}

int skb_engine_view(skb_engine* e, int which, void** ptr, int64_t* numel) {
    if (!e || !ptr || !numel) return fail(SKB_ERR_ARG, "view: null argument");
    switch (which) {
        case 0: *ptr = e->x; *numel = (int64_t)e->R * e->D; break;
        case 1: *ptr = e->hidden; *numel = (int64_t)e->R * e->D; break;
        case 2: *ptr = e->logits; *numel = (int64_t)e->R * e->V; break;
        case 3: *ptr = e->pos; *numel = e->R; break;
        case 4: *ptr = e->logits_hist; *numel = (int64_t)e->Q * e->R * e->V; break;
        case 5: *ptr = e->prefix; *numel = (int64_t)e->nreq * e->D; break;
        case 6: *ptr = e->err; *numel = 8; break;
        case 7: *ptr = e->st; *numel = (int64_t)e->nreq * (int64_t)(sizeof(ReqState) / 4); break;
        case 8: *ptr = e->kts; *numel = (int64_t)SKB_KTS_STRIDE * kts_slots(e); break;
        case 9: *ptr = e->dh_ts; *numel = (int64_t)2 * depth_head_phases(e->Q); break;
        default: return fail(SKB_ERR_ARG, "view: unknown buffer %d", which);
    }
    return SKB_OK;
}

int skb_engine_set_debug(skb_engine* e, int on) {
    if (!e) return fail(SKB_ERR_ARG, "set_debug: null engine");
    if ((on != 0) != (e->debug != 0)) destroy_graph(e);
    e->debug = on != 0;
    return SKB_OK;
}

int skb_engine_kernels_per_frame(skb_engine* e) {
    if (!e) return -1;
    return e->frame_nodes > 0 ? e->frame_nodes : e->Q * 4 + e->L * 5;
}

int skb_engine_launches_per_step(skb_engine* e) {
    if (!e) return -1;
    if (!e->exec) return 0;
    return e->graph_fpg * skb_engine_kernels_per_frame(e);
}

}  // extern "C"
