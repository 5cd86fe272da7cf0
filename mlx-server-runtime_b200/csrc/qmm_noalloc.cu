// mlxq_quantized_matmul_noalloc: quantized_matmul for callers that cannot allocate
// device memory (see include/mlxq_b200.h). The K-split scratch of the decode
// kernel lives in a fixed array in this library's device image instead of a
// caller workspace.
#include <atomic>
#include <cstdio>
#include <mutex>

#include "../../include/mlxq_b200.h"
#include "launch.h"

namespace {

// Scratch for K-split partial sums and row-block tickets, shared by every call
// on a device. Every GPU that loads the library holds it until the process exits.
constexpr size_t kScratchBytes = MLXQ_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
// Per-device launch limits and the device address of g_scratch. A device's entry
// is filled once under g_setup_mu; g_scratch_ptr is stored last with release
// order, so a thread that loads a non-null pointer (acquire) also sees the limits.
struct DeviceSetup {
    int num_sms = 0;
    int max_smem = 0;
};
DeviceSetup g_setup[kMaxDevices];
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mu;

int fail(int code, const char* fmt, long long a = 0, long long b = 0) {
    char buf[256];
    snprintf(buf, sizeof(buf), fmt, a, b);
    return mlxq::set_last_error(code, buf);
}

int cuda_fail(cudaError_t e, const char* what) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    return mlxq::set_last_error(MLXQ_ERR_CUDA, buf);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Once per device, with that device current: the device address of the scratch
// array (the host-side symbol is only a stand-in) and the launch limits. Host
// threads making a device's first call at the same time serialize on the mutex.
int setup_device(int dev, void** scratch) {
    void* ready = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (ready != nullptr) {
        *scratch = ready;
        return MLXQ_OK;
    }
    std::lock_guard<std::mutex> lock(g_setup_mu);
    ready = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (ready != nullptr) {
        *scratch = ready;
        return MLXQ_OK;
    }
    int sms = 0, smem = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
    e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
    g_setup[dev].num_sms = sms;
    g_setup[dev].max_smem = smem - 1024;
    g_scratch_ptr[dev].store(ptr, std::memory_order_release);
    *scratch = ptr;
    return MLXQ_OK;
}

}  // namespace

extern "C" int mlxq_quantized_matmul_noalloc(const void* x, const uint32_t* w, const void* scales,
                                             const void* biases, const void* bias, void* out,
                                             int64_t M, int64_t N, int64_t K, int group_size,
                                             int bits, int dtype, void* stream) {
    if (bits != 4 && bits != 8)
        return fail(MLXQ_ERR_UNSUPPORTED_BITS, "bits=%lld is not supported (4 or 8)", bits);
    if (group_size != 32 && group_size != 64 && group_size != 128)
        return fail(MLXQ_ERR_GROUP_SIZE, "group_size=%lld is not one of 32, 64, 128", group_size);
    if (K <= 0 || K % group_size != 0)
        return fail(MLXQ_ERR_SHAPE, "K=%lld must be a positive multiple of group_size=%lld", K,
                    group_size);
    if (M < 0 || N <= 0 || M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
        return fail(MLXQ_ERR_SHAPE, "quantized_matmul_noalloc: bad shape M=%lld N=%lld", M, N);
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "quantized_matmul_noalloc: dtype=%lld must be bf16 or f16",
                    dtype);
    if (!x || !w || !scales || !biases || !out)
        return fail(MLXQ_ERR_NULL, "quantized_matmul_noalloc: NULL pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases) ||
        !aligned16(out) || (bias && !aligned16(bias)))
        return fail(MLXQ_ERR_ALIGN, "quantized_matmul_noalloc: pointers must be 16-byte aligned");
    if (M == 0) return MLXQ_OK;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(MLXQ_ERR_CUDA, "device %lld out of range", dev);
    void* scratch = nullptr;
    int rc = setup_device(dev, &scratch);
    if (rc) return rc;

    mlxq::QmvPlan plan;
    if (!mlxq::qmv_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                        static_cast<int>(K), 0, 0, g_setup[dev].num_sms, g_setup[dev].max_smem,
                        &plan))
        return fail(MLXQ_ERR_SHAPE, "quantized_matmul_noalloc: no launch plan fits shared memory");
    // This entry point's scratch layout: the tickets (one per row block and token
    // tile), rounded up to 256 bytes, then the fp32 partial sums of every K split.
    const size_t counters = static_cast<size_t>(plan.ztotal) * plan.rowblocks * 4;
    const size_t need = plan.splits > 1
                            ? (counters + 255) / 256 * 256 +
                                  static_cast<size_t>(plan.splits) * M * static_cast<size_t>(N) * 4
                            : 0;
    if (need > kScratchBytes)
        return fail(MLXQ_ERR_WORKSPACE,
                    "quantized_matmul_noalloc: this shape needs %lld bytes of scratch but the "
                    "built-in scratch holds %lld; use mlxq_quantized_matmul with a workspace",
                    static_cast<long long>(need), static_cast<long long>(kScratchBytes));

    mlxq::QmvParams p{};
    p.x = x; p.w = w; p.s = scales; p.b = biases; p.bias = bias; p.out = out;
    p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
    p.mode = 0; p.lhs = nullptr; p.lhs_div = 1; p.rhs = nullptr; p.seg = nullptr;
    p.batch = 0; p.num_experts = 1; p.x_batches = 1; p.w_estride = 0; p.sb_estride = 0;
    p.splits = plan.splits; p.gps = plan.gps; p.win = plan.win; p.ztotal = plan.ztotal;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (need > 0) {
        // The tickets must start at zero: the array keeps whatever the last call left.
        char* base = static_cast<char*>(scratch);
        e = cudaMemsetAsync(base, 0, counters, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch tickets)");
        p.counter = reinterpret_cast<unsigned*>(base);
        p.partial = reinterpret_cast<float*>(base + (counters + 255) / 256 * 256);
    }
    plan.overlap = false;
    e = mlxq::qmv_launch(dtype, bits, group_size, plan, p, st);
    if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul_noalloc launch");
    return MLXQ_OK;
}
