// Persistent frame kernel: program description and host entry points.
#pragma once

#include "engine_types.cuh"
#include "gemv.cuh"
#include "trunk.cuh"

namespace skb {

constexpr int FK_CONSUMER_THREADS = 256;  // 8 consumer warps
constexpr int FK_THREADS = 288;           // + 1 producer warp
constexpr int FK_SLOTS = 6;
constexpr uint32_t FK_SLOT_BYTES = 24 * 1024;
constexpr int FK_VMAX = 2304;  // audio vocabulary capacity of the in-kernel sampler
constexpr size_t FK_HEAD = 256;
constexpr size_t FK_SMEM = FK_HEAD + (size_t)FK_SLOTS * FK_SLOT_BYTES + sampler_smem_bytes<FK_VMAX>();

enum : int { PH_GEMV = 0, PH_ATTN = 1 };

// One phase of the frame program.  GEMV phases carry the same arguments a
// gemv_kernel launch takes; `sample` marks the classifier phase whose last
// CTA runs the depth sampler for the first n_req requests.
struct Phase {
    int kind;
    int xm, em, kv4;
    int sample;
    int n_req;
    int attn_rows;
    GemvArgs g;
    DepthSampleArgs s;
    DecodeAttnArgs at;
};

struct FrameArgs {
    const Phase* prog;
    int n_phases;
    int frames;
    unsigned* bar_count;  // grid-barrier arrivals, zeroed before each launch
    int* abort_flag;      // raised by any timeout; every CTA stops
    int* err;             // err[2]: copy wait timed out / bad phase; err[3]: grid barrier timed out
    int* sample_ticket;   // classifier-phase ticket (left at zero)
    unsigned long long* timeline;  // optional [frames * n_phases * 2]: CTA 0's phase start and
                                   // end (%globaltimer ns); the sampler CTA overwrites the end of
                                   // a classifier phase with the time its sampling finished
    unsigned long long* cta_end;   // optional [frames * n_phases * gridDim]: each CTA's phase end
};

size_t frame_kernel_smem();
cudaError_t frame_kernel_prepare(int M);
int frame_kernel_occupancy(int M);
cudaError_t frame_kernel_launch(int M, const FrameArgs& fa, int grid, cudaStream_t s);

}  // namespace skb
