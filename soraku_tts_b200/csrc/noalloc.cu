// skb_decode_attention_noalloc: decode attention whose scratch lives in a
// library-owned device array, for callers that cannot allocate device memory
// while decoding (see the declaration in include/soraku_b200.h for who they are
// and why).
//
// The array is a file-scope __device__ variable.  In host code its name is
// only a host-side stand-in, not a device address: handing it to a kernel
// would fault, or read the wrong memory.  So the first call on each device
// looks the device address up with cudaGetSymbolAddress while that device is
// current, checks the result and caches it; every launch receives that looked-up
// pointer.  The cached address belongs to the device's current context: after
// cudaDeviceReset on that device it is stale, so a program that resets a
// device must not call this entry point on it again.  Every call reuses the
// array, which keeps the previous call's contents: the tickets, which must
// start at zero, are cleared with cudaMemsetAsync on the caller's stream
// before each launch (after every argument check).  Calls that overlap on the
// GPU share the array and therefore race.
#include <mutex>

#include "ops.cuh"
#include "trunk_api.cuh"

// [tickets (1 KiB) | split partials (2 MiB)]
static constexpr size_t kNoallocTicketBytes = 1024;
static constexpr size_t kNoallocPartBytes = 2u * 1024u * 1024u;
static_assert(kNoallocTicketBytes + kNoallocPartBytes == SKB_NOALLOC_SCRATCH_BYTES,
              "header and library disagree on the scratch size");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocTicketBytes + kNoallocPartBytes];

namespace skb {

int decode_attention_check(const float* qkv, int rows, int H, int KVH, int hd, const float* qn, const float* kn,
                           const float* rc, const float* rs, int max_len, const int32_t* pos, const float* kv_pool,
                           const int32_t* page_table, int max_pages, int page_size, int n_pages, int splits,
                           const float* out);
int decode_attention_op(const float* qkv, int rows, int H, int KVH, int hd, const float* qn, const float* kn,
                        float eps, const float* rc, const float* rs, int max_len, const int32_t* pos, float* kv_pool,
                        const int32_t* page_table, int max_pages, int page_size, int n_pages, int splits,
                        float* part, int32_t* tickets, float* out, cudaStream_t stream);

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_for_current_device(unsigned char** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return fail(SKB_ERR_CUDA, "decode_attention_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(SKB_ERR_ARG, "decode_attention_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // device `dev` is current
        if (e != cudaSuccess || p == nullptr)
            return fail(SKB_ERR_CUDA, "decode_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
    return SKB_OK;
}

}  // namespace
}  // namespace skb

extern "C" int skb_decode_attention_noalloc(const float* qkv, int rows, int n_heads, int n_kv_heads, int head_dim,
                                            const float* q_norm, const float* k_norm, float eps,
                                            const float* rope_cos, const float* rope_sin, int max_len,
                                            const int32_t* pos, float* kv_pool, const int32_t* page_table,
                                            int max_pages, int page_size, int n_pages, int splits, float* out,
                                            cudaStream_t stream) {
    using namespace skb;
    if (rows < 1 || n_kv_heads < 1 || splits < 1 || head_dim < 1 || n_heads < n_kv_heads)
        return fail(SKB_ERR_ARG, "decode_attention_noalloc: bad sizes");
    const unsigned long long n_rep = (unsigned long long)(n_heads / n_kv_heads);
    const unsigned long long tickets = (unsigned long long)rows * n_kv_heads;
    const unsigned long long part_floats =
        tickets * (unsigned long long)splits * n_rep * (unsigned long long)(head_dim + 2);
    if (tickets * 4 > kNoallocTicketBytes || part_floats * 4 > kNoallocPartBytes)
        return fail(SKB_ERR_ARG,
                    "decode_attention_noalloc: rows %d x kv heads %d x splits %d needs %llu bytes of partials "
                    "and %llu of tickets; the built-in scratch holds %zu and %zu",
                    rows, n_kv_heads, splits, part_floats * 4, tickets * 4, kNoallocPartBytes, kNoallocTicketBytes);
    // every argument is checked before the shared array is touched, so a
    // rejected call never disturbs a call still running on another stream
    const int chk = decode_attention_check(qkv, rows, n_heads, n_kv_heads, head_dim, q_norm, k_norm, rope_cos,
                                           rope_sin, max_len, pos, kv_pool, page_table, max_pages, page_size,
                                           n_pages, splits, out);
    if (chk != SKB_OK) return chk;
    unsigned char* scratch = nullptr;
    const int st = scratch_for_current_device(&scratch);
    if (st != SKB_OK) return st;
    int32_t* tk = reinterpret_cast<int32_t*>(scratch);
    float* part = reinterpret_cast<float*>(scratch + kNoallocTicketBytes);
    const cudaError_t e = cudaMemsetAsync(tk, 0, tickets * 4, stream);
    if (e != cudaSuccess)
        return fail(SKB_ERR_CUDA, "decode_attention_noalloc: clearing tickets: %s", cudaGetErrorString(e));
    return decode_attention_op(qkv, rows, n_heads, n_kv_heads, head_dim, q_norm, k_norm, eps, rope_cos, rope_sin,
                               max_len, pos, kv_pool, page_table, max_pages, page_size, n_pages, splits, part, tk,
                               out, stream);
}
