// Host-side launcher declarations shared by the C-ABI layer (abi.cu) and the
// kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace mlxq {

// Serializes the one-time per-device setup calls of every launcher (abi.cu).
std::mutex& setup_mutex();

// Per-device record of a value set up once (a kernel's dynamic shared-memory
// limit, an SM count): zero until set, only ever raised, published with release
// order so a thread that reads it also sees what was done before.
struct PerDevice {
    std::atomic<int> v[64];
};

// Raises `kern`'s dynamic shared-memory limit on the current device `dev` to at
// least `smem` (never lowers it); host threads racing on a first launch serialize.
// The kernel's preferred carveout is set to the whole shared-memory capacity at the
// same time. The SM's L1/shared split otherwise follows each kernel's own size
// (e.g. 132 KB for one 104 KB CTA), and an SM configured for one split has to drain
// before it takes a CTA that needs another: back-to-back kernels with different
// needs could then never share an SM, and launch overlap would not overlap.
template <typename K>
cudaError_t ensure_smem_attr(K kern, PerDevice& cache, int dev, int smem) {
    if (cache.v[dev].load(std::memory_order_acquire) >= smem) return cudaSuccess;
    std::lock_guard<std::mutex> lock(setup_mutex());
    const int have = cache.v[dev].load(std::memory_order_relaxed);
    if (have >= smem) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (have == 0) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
    }
    cache.v[dev].store(smem, std::memory_order_release);
    return cudaSuccess;
}

// The carveout part of ensure_smem_attr alone, for kernels with no dynamic shared
// memory above the default limit.
template <typename K>
cudaError_t ensure_carveout(K kern, PerDevice& cache, int dev) {
    return ensure_smem_attr(kern, cache, dev, 1);
}

// The calling thread's current device, checked against the per-device tables.
inline cudaError_t current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return e;
    return (*dev < 0 || *dev >= 64) ? cudaErrorInvalidDevice : cudaSuccess;
}

enum { kF32 = 0, kBF16 = 1, kF16 = 2 };

// Layout of the quantized_matmul workspace shared by the decode kernels: a fixed
// ticket region (one counter per row block, zero between calls) followed by the
// fp32 partial sums of the current call. The ticket region never moves, so
// partial sums written by one call can never land where a later call, planned
// with more row blocks, expects zeroed tickets.
constexpr size_t kTicketBytes = 64 * 1024;
// The last 256 bytes of the ticket region hold the fused greedy argmax's done counter
// and per-token keys (zero between calls, like the tickets); tickets stay below it.
constexpr size_t kArgmaxOffset = kTicketBytes - 256;

cudaError_t launch_quantize(const void* w, int dtype, uint32_t* wq, void* s, void* b,
                            long long rows, long long K, int gs, int bits, cudaStream_t st);
cudaError_t launch_dequantize(const uint32_t* wq, const void* s, const void* b, int dtype,
                              void* out, long long rows, long long K, int gs, int bits,
                              cudaStream_t st);

// One problem for the skinny (decode) tensor-core kernel family.
//   mode 0: dense  out[M,N] = x[M,K] @ W^T
//   mode 1: gather, one batch entry per grid z: out[b] = x[xi(b)] @ W[rhs[b]]^T
//   mode 2: gather with rhs sorted; grid z = expert, rows of expert e are the
//           batch entries [seg[e], seg[e+1]) of a segment table built on device.
struct QmvParams {
    const void* x;
    const uint32_t* w;
    const void* s;
    const void* b;
    const void* bias;  // optional per-output bias [N] (mode 0 only)
    void* out;
    int M, N, K;
    int mode;
    const int32_t* lhs;  // optional x-batch index per batch entry
    int lhs_div;         // xi(b) = b / lhs_div when lhs == nullptr
    const int32_t* rhs;  // expert per batch entry
    const int32_t* seg;  // mode 2: [num_experts + 1] row offsets
    int batch;
    int num_experts;
    int x_batches;         // number of [M, K] matrices x holds (gather modes)
    long long w_estride;   // words per expert
    long long sb_estride;  // scale/bias elements per expert
    int splits;            // K splits (mode 0)
    int gps;               // groups per split
    int win;               // groups per shared-memory window (multiple of the chunk)
    int ztotal;            // number of z work items
    float* partial;        // [splits][M][N] fp32, used when splits > 1
    unsigned* counter;     // [ztotal][gridDim.x], zero at entry and exit
};

struct QmvPlan {
    int nt;       // n-tiles of 8 tokens (1, 2 or 4)
    int splits;
    int gps;
    int win;
    int rowblocks;
    int ztotal;
    int gridz;
    size_t smem;
    bool sbvec;
    bool single;   // one token per pass (selects the kernel without odd-column folds)
    bool overlap;  // launch with programmatic stream serialization (launch overlap)
    size_t ws_bytes;  // workspace the plan needs (0 if none)
};

// Plans and launches the skinny kernel (defined in qmv_dispatch.cu).
bool qmv_plan(int dtype, int bits, int gs, int M_tokens_per_item, int N, int K, int mode,
              int z_items, int num_sms, int max_smem, QmvPlan* plan);
cudaError_t qmv_launch(int dtype, int bits, int gs, const QmvPlan& plan, const QmvParams& p,
                       cudaStream_t st);

// Plan of the TMA-fed decode kernel (qmv_tma.cu): M <= 8 tokens, K/group_size a
// multiple of 8. Units of BR rows x 8 groups, split evenly over P CTAs. Epilogue `epi`:
// 0 the outputs; 1 silu(gate) * up from a gate/up-interleaved w (N % 16 == 0, no bias);
// 2 the greedy argmax over N per token into int32 out[M] (workspace required).
struct QtPlan {
    int BR;        // rows per unit (64 or 16)
    int RB;        // row blocks of BR rows
    int S;         // units per row block
    long long U;   // units
    int P;         // CTAs
    int GL;        // most K groups one CTA stages activations for
    int stages;    // ring depth
    int maxc;      // most CTAs sharing one row block
    bool heads;    // a ticket warp takes the head row blocks' tickets (64-row units)
    size_t smem;
    size_t ws_bytes;  // workspace (tickets + partials) when a row block is shared
};
bool qmv_tma_plan(int dtype, int bits, int gs, int M, int N, int K, int num_sms, int max_smem,
                  int sm_smem, QtPlan* plan);
cudaError_t qmv_tma_launch(int dtype, int bits, int gs, const QtPlan& plan, const void* x,
                           const uint32_t* w, const void* s, const void* b, const void* bias,
                           void* out, int M, int N, int K, void* workspace, bool overlap,
                           cudaStream_t st, int epi = 0);
cudaError_t qmv_tma_read_error(int* out_code);

// One problem for the TMA-fed grouped decode kernel (qmv_grouped.cu): gather_qmm
// entries b (expert rhs[b], x entry lhs[b] or b / lhs_div, M rows each) against
// experts' weights stacked [E, N, ...]. sorted: rhs is non-decreasing and entry b's
// x rows are entry b's (no lhs, x_batches == batch), so an expert's rows are taken
// together, TM at a time.
struct QgdPlan {
    int TM;        // token slots of a chunk
    int BR;        // weight rows per item
    int S;         // 8-group stages per item
    int RB;        // row blocks of N
    int P;         // CTAs
    int stages;    // ring depth
    bool sorted;
    size_t smem;
};
bool qmv_grouped_plan(int bits, int gs, long long batch, int M, int N, int K, int E, bool sorted,
                      int num_sms, int max_smem, int sm_smem, QgdPlan* plan);
cudaError_t qmv_grouped_launch(int dtype, int bits, int gs, const QgdPlan& plan, const void* x,
                               const uint32_t* w, const void* s, const void* b, void* out,
                               const int32_t* rhs, const int32_t* lhs, int lhs_div, int batch,
                               int x_batches, int M, int N, int K, int E, bool overlap,
                               cudaStream_t st, int epi = 0);
// A single bounded wait that runs out (mlxq_check_bounded_wait).
cudaError_t launch_bounded_wait_check(uint32_t polls, cudaStream_t st);

// One problem for the tcgen05 prefill kernel (qgemm_sm100.cu): dense, or grouped by
// expert (sorted gather_qmm) when E > 0: rows [seg[e]*rpe, seg[e+1]*rpe) of x and out
// use expert e's weights (w, s, b hold E stacked [N, ...] matrices); tile_start[e]
// is the first output tile of expert e and tile_start[E] the tile count.
struct QgemmParams {
    const void* x;
    const uint32_t* w;
    const void* s;
    const void* b;
    const void* bias;  // optional per-output bias [N] (dense only)
    void* out;
    int M, N, K;       // M: rows of x and out (all experts' rows when grouped)
    int E;             // 0: dense
    int rpe;           // rows per batch entry (grouped)
    const int32_t* seg;
    const int32_t* tile_start;
    int sk;            // stream-K (dense only): CTAs take equal shares of tiles x K blocks
    unsigned* counter; // stream-K tickets, one per tile, zero at entry and exit
    float* partial;    // stream-K fp32 partial tiles, two slots per CTA
    int narrow;        // dense whole tiles of 128 tokens instead of 192 (more tiles)
    int grid;          // stream-K CTAs (0: one per SM)
    int epi;           // 1: SwiGLU over gate/up rows interleaved by 16-row tiles (dense
                       // whole tiles), out [M, N / 2]
};

// Plan of the prefill kernel for a dense problem: data-parallel whole tiles, or
// stream-K when whole tiles would leave a large part of the last wave idle.
struct QgemmPlan {
    bool stream_k;
    bool narrow;      // whole tiles of 128 tokens: more tiles for a shape that has few
    int grid;         // stream-K CTAs: one per SM, or fewer when K is short
    size_t ws_bytes;  // workspace (tickets + partial tiles) for stream-K, else 0
};
bool qgemm_plan(int M, int N, int K, int num_sms, QgemmPlan* plan);

bool qgemm_supported(int M, int N, int K, int bits, int gs);
// Builds tile_start[0..E] for a grouped problem from seg (qgemm_sm100.cu).
cudaError_t launch_group_tiles(const int32_t* seg, int E, int rpe, int N, int32_t* tile_start,
                               cudaStream_t st);
cudaError_t qgemm_launch(int dtype, int bits, int gs, const QgemmParams& p, cudaStream_t st);
// Reads (and clears) the error code a kernel recorded after a bounded wait gave up.
cudaError_t qgemm_read_error(int* out_code);

// Process-wide launch-overlap switch (mlxq_set_launch_overlap).
bool launch_overlap_enabled();

// Sets the thread's mlxq_last_error() message and returns `code`.
int set_last_error(int code, const char* msg);

cudaError_t launch_segments(const int32_t* rhs, int batch, int num_experts, int32_t* seg,
                            cudaStream_t st);

}  // namespace mlxq
