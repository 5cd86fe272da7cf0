// extern "C" entry points of libmlxq_b200.so (declared in include/mlxq_b200.h).
// Host-side validation happens before anything is enqueued; every failure
// returns a negative code and records a message for mlxq_last_error().
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mlxq_b200.h"
#include "launch.h"

namespace {

thread_local std::string g_last_error;
std::atomic<int> g_overlap{0};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(MLXQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct DeviceInfo {
    int num_sms = 0;
    int max_smem = 0;  // usable dynamic shared memory per CTA
    int sm_smem = 0;   // shared memory per SM
};

// Properties of the calling thread's current device (cached per device: filled once
// under the setup mutex, published by a release store of `ready`).
int device_info(DeviceInfo* out, cudaStream_t stream) {
    static DeviceInfo cache[64];
    static std::atomic<int> ready[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
#if CUDART_VERSION >= 12080
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (stream != nullptr) e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    // cudaStreamGetDevice is not permitted on a capturing stream; the check is
    // skipped while a graph is being captured.
    if (stream != nullptr && cap == cudaStreamCaptureStatusNone) {
        int sdev = -1;
        e = cudaStreamGetDevice(stream, &sdev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamGetDevice");
        if (sdev != dev)
            return fail(MLXQ_ERR_CUDA, "stream belongs to device %d but device %d is current",
                        sdev, dev);
    }
#else
    (void)stream;
#endif
    if (dev < 0 || dev >= 64) return fail(MLXQ_ERR_CUDA, "device ordinal %d out of range", dev);
    if (!ready[dev].load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(mlxq::setup_mutex());
        if (ready[dev].load(std::memory_order_relaxed)) {
            *out = cache[dev];
            return MLXQ_OK;
        }
        int sms = 0, smem = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
        e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
        int sm_smem = 0;
        e = cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem per SM)");
        cache[dev].max_smem = smem - 1024;  // room for the kernels' static shared memory
        cache[dev].sm_smem = sm_smem;
        cache[dev].num_sms = sms;
        ready[dev].store(1, std::memory_order_release);
    }
    *out = cache[dev];
    return MLXQ_OK;
}

int check_bits_gs(int bits, int group_size, bool matmul) {
    const bool bits_ok = matmul ? (bits == 4 || bits == 8) : (bits == 2 || bits == 4 || bits == 8);
    if (!bits_ok)
        return fail(MLXQ_ERR_UNSUPPORTED_BITS, "bits=%d is not supported (%s)", bits,
                    matmul ? "4 or 8" : "2, 4 or 8");
    if (group_size != 32 && group_size != 64 && group_size != 128)
        return fail(MLXQ_ERR_GROUP_SIZE, "group_size=%d is not one of 32, 64, 128", group_size);
    return MLXQ_OK;
}

int check_k(int64_t K, int group_size) {
    if (K <= 0 || K % group_size != 0)
        return fail(MLXQ_ERR_SHAPE, "K=%lld must be a positive multiple of group_size=%d",
                    static_cast<long long>(K), group_size);
    return MLXQ_OK;
}

constexpr int64_t kIntMax = 0x7fffffffLL;
// Sorted gather_qmm goes to the grouped tensor-core kernel from this many rows per
// expert on average (below it, the weight-streaming decode kernel is as fast).
constexpr int64_t kGroupedMinRows = 24;

size_t dense_plan(int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
                  const DeviceInfo& di, mlxq::QmvPlan* plan, bool* ok) {
    *ok = mlxq::qmv_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                         static_cast<int>(K), 0, 0, di.num_sms, di.max_smem, plan);
    return *ok ? plan->ws_bytes : 0;
}

}  // namespace

namespace mlxq {
bool launch_overlap_enabled() { return g_overlap.load(std::memory_order_relaxed) != 0; }

std::mutex& setup_mutex() {
    static std::mutex mu;
    return mu;
}

// Records the message mlxq_last_error() returns; for entry points defined in
// other translation units.
int set_last_error(int code, const char* msg) {
    g_last_error = msg;
    return code;
}
}  // namespace mlxq

extern "C" {

int mlxq_set_launch_overlap(int enable) {
    const int prev = g_overlap.exchange(enable ? 1 : 0);
    return prev;
}

int mlxq_get_launch_overlap(void) { return g_overlap.load(); }

int mlxq_device_error(int* code) {
    if (!code) return fail(MLXQ_ERR_NULL, "device_error: NULL pointer");
    *code = 0;
    int a = 0, b = 0;
    cudaError_t e = mlxq::qgemm_read_error(&a);
    if (e == cudaSuccess) e = mlxq::qmv_tma_read_error(&b);
    if (e != cudaSuccess) return cuda_fail(e, "device_error");
    *code = a ? a : b;
    return MLXQ_OK;
}

int mlxq_check_bounded_wait(uint32_t polls, void* stream) {
    if (polls == 0 || polls > (1u << 22))
        return fail(MLXQ_ERR_SHAPE, "check_bounded_wait: polls=%u must be in [1, 2^22]", polls);
    cudaError_t e = mlxq::launch_bounded_wait_check(polls, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "check_bounded_wait launch");
    return MLXQ_OK;
}

int mlxq_abi_version(void) { return MLXQ_ABI_VERSION; }

const char* mlxq_last_error(void) { return g_last_error.c_str(); }

int mlxq_quantize(const void* w, int w_dtype, uint32_t* wq, void* scales, void* biases,
                  int64_t rows, int64_t K, int group_size, int bits, void* stream) {
    int rc = check_bits_gs(bits, group_size, false);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (rows < 0) return fail(MLXQ_ERR_SHAPE, "rows=%lld must be >= 0", (long long)rows);
    if (w_dtype != MLXQ_F32 && w_dtype != MLXQ_BF16 && w_dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "w_dtype=%d is not float32, bfloat16 or float16", w_dtype);
    if (!w || !wq || !scales || !biases) return fail(MLXQ_ERR_NULL, "quantize: NULL pointer");
    if (!aligned16(w) || !aligned16(wq) || !aligned16(scales) || !aligned16(biases))
        return fail(MLXQ_ERR_ALIGN, "quantize: pointers must be 16-byte aligned");
    if (rows == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_quantize(w, w_dtype, wq, scales, biases, rows, K, group_size, bits,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    return MLXQ_OK;
}

int mlxq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int dtype,
                    void* out, int64_t rows, int64_t K, int group_size, int bits, void* stream) {
    int rc = check_bits_gs(bits, group_size, false);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (rows < 0) return fail(MLXQ_ERR_SHAPE, "rows=%lld must be >= 0", (long long)rows);
    if (dtype != MLXQ_F32 && dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "dtype=%d is not float32, bfloat16 or float16", dtype);
    if (!wq || !scales || !biases || !out) return fail(MLXQ_ERR_NULL, "dequantize: NULL pointer");
    if (!aligned16(wq) || !aligned16(scales) || !aligned16(biases) || !aligned16(out))
        return fail(MLXQ_ERR_ALIGN, "dequantize: pointers must be 16-byte aligned");
    if (rows == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_dequantize(wq, scales, biases, dtype, out, rows, K, group_size,
                                            bits, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
    return MLXQ_OK;
}

// Rows the TMA-fed decode kernel takes in one launch (its token slots). 17-32 rows of a
// small matrix run as two launches of it (rows 0-15, then the rest): each launch
// streams the weights again, which pays only while they are small (k/v 512x3584 at 32
// rows: 16.8 us against 30.1 us on the cp.async kernel; gate/up 18944x3584: 37.9 us
// against 28.1 us). MLXQ_DECODE_CHUNKS=0 (read once per process) turns it off, for
// comparisons.
constexpr int64_t kTmaRows = 16;
constexpr int64_t kChunkMaxWeightBytes = 4 << 20;

static bool decode_chunks_enabled() {
    static const bool v = [] {
        const char* e = std::getenv("MLXQ_DECODE_CHUNKS");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return v;
}

// Plans of the (at most two) row chunks of a decode-sized quantized_matmul on the TMA
// kernel: plan[0] for the first kTmaRows rows (or all of M), plan[1] for the rest
// (a copy of plan[0] when M <= kTmaRows). False when the kernel does not take the shape.
static bool tma_row_chunks(int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
                           const DeviceInfo& di, mlxq::QtPlan plan[2]) {
    if (M < 1 || M > 2 * kTmaRows) return false;
    if (M > kTmaRows && (!decode_chunks_enabled() || N * K * bits / 8 > kChunkMaxWeightBytes))
        return false;
    const int64_t m0 = std::min(M, kTmaRows);
    if (!mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(m0), static_cast<int>(N),
                            static_cast<int>(K), di.num_sms, di.max_smem, di.sm_smem, &plan[0]))
        return false;
    plan[1] = plan[0];
    if (M > kTmaRows &&
        !mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(M - kTmaRows),
                            static_cast<int>(N), static_cast<int>(K), di.num_sms, di.max_smem,
                            di.sm_smem, &plan[1]))
        return false;
    return true;
}

size_t mlxq_qmm_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits,
                               int dtype) {
    if (check_bits_gs(bits, group_size, true) || check_k(K, group_size)) return 0;
    if (M <= 0 || N <= 0 || M > kIntMax || N > kIntMax || K > kIntMax) return 0;
    DeviceInfo di;
    if (device_info(&di, nullptr)) return 0;
    if (mlxq::qgemm_supported(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                              bits, group_size)) {
        // the tensor-core prefill kernel: tickets + partial tiles when it runs stream-K
        mlxq::QgemmPlan gp;
        mlxq::qgemm_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                         di.num_sms, &gp);
        return gp.ws_bytes;
    }
    mlxq::QtPlan tplan[2];
    if (tma_row_chunks(M, N, K, group_size, bits, dtype, di, tplan))
        return std::max(tplan[0].ws_bytes, tplan[1].ws_bytes);
    mlxq::QmvPlan plan;
    bool ok = false;
    return dense_plan(M, N, K, group_size, bits, dtype, di, &plan, &ok);
}

int mlxq_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                          const void* biases, const void* bias, void* out, int64_t M, int64_t N,
                          int64_t K, int group_size, int bits, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
    int rc = check_bits_gs(bits, group_size, true);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (M < 0 || N <= 0 || M > kIntMax || N > kIntMax || K > kIntMax)
        return fail(MLXQ_ERR_SHAPE, "quantized_matmul: bad shape M=%lld N=%lld K=%lld",
                    (long long)M, (long long)N, (long long)K);
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "quantized_matmul: dtype=%d must be bfloat16 or float16", dtype);
    if (!x || !w || !scales || !biases || !out)
        return fail(MLXQ_ERR_NULL, "quantized_matmul: NULL pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases) ||
        !aligned16(out) || (bias && !aligned16(bias)))
        return fail(MLXQ_ERR_ALIGN, "quantized_matmul: pointers must be 16-byte aligned");
    if (M == 0) return MLXQ_OK;
    DeviceInfo di;
    if ((rc = device_info(&di, static_cast<cudaStream_t>(stream)))) return rc;
    if (mlxq::qgemm_supported(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), bits,
                              group_size)) {
        // prefill: dequantize into tensor memory + tcgen05 tensor cores
        mlxq::QgemmParams q{};
        q.x = x; q.w = w; q.s = scales; q.b = biases; q.bias = bias; q.out = out;
        q.M = static_cast<int>(M); q.N = static_cast<int>(N); q.K = static_cast<int>(K);
        // Stream-K (shapes whose whole tiles leave much of the last wave idle) needs the
        // workspace; without one (or too small) the kernel runs whole tiles instead.
        mlxq::QgemmPlan gp;
        mlxq::qgemm_plan(q.M, q.N, q.K, di.num_sms, &gp);
        q.narrow = gp.narrow ? 1 : 0;
        if (gp.stream_k && workspace && workspace_bytes >= gp.ws_bytes &&
            !(reinterpret_cast<uintptr_t>(workspace) & 255u)) {
            q.sk = 1;
            q.grid = gp.grid;
            q.counter = static_cast<unsigned*>(workspace);
            q.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + mlxq::kTicketBytes);
        } else if (gp.stream_k && gp.grid < di.num_sms) {
            // a short-K shape with few tiles and no room for its partials: 128-token
            // tiles, more of them than 192-token ones
            q.narrow = (M + 127) / 128 > (M + 191) / 192 ? 1 : 0;
        }
        cudaError_t e = mlxq::qgemm_launch(dtype, bits, group_size, q,
                                           static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul (prefill) launch");
        return MLXQ_OK;
    }
    mlxq::QtPlan tplan[2];
    if (tma_row_chunks(M, N, K, group_size, bits, dtype, di, tplan)) {
        // decode, M <= 32: the TMA-fed stream-K kernel, 16 rows per launch
        const size_t need = std::max(tplan[0].ws_bytes, tplan[1].ws_bytes);
        if (need > 0) {
            if (!workspace || workspace_bytes < need)
                return fail(MLXQ_ERR_WORKSPACE,
                            "quantized_matmul: needs %zu workspace bytes, got %zu", need,
                            workspace ? workspace_bytes : (size_t)0);
            if (reinterpret_cast<uintptr_t>(workspace) & 255u)
                return fail(MLXQ_ERR_ALIGN, "quantized_matmul: workspace must be 256-byte aligned");
        }
        for (int64_t r0 = 0, c = 0; r0 < M; r0 += kTmaRows, ++c) {
            const int64_t mc = std::min(kTmaRows, M - r0);
            cudaError_t e = mlxq::qmv_tma_launch(
                dtype, bits, group_size, tplan[c], static_cast<const char*>(x) + r0 * K * 2, w,
                scales, biases, bias, static_cast<char*>(out) + r0 * N * 2,
                static_cast<int>(mc), static_cast<int>(N), static_cast<int>(K), workspace,
                mlxq::launch_overlap_enabled(), static_cast<cudaStream_t>(stream));
            if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul (decode) launch");
        }
        return MLXQ_OK;
    }
    mlxq::QmvPlan plan;
    bool ok = false;
    const size_t need = dense_plan(M, N, K, group_size, bits, dtype, di, &plan, &ok);
    if (!ok) return fail(MLXQ_ERR_SHAPE, "quantized_matmul: no launch plan fits shared memory");
    if (need > 0) {
        if (!workspace || workspace_bytes < need)
            return fail(MLXQ_ERR_WORKSPACE, "quantized_matmul: needs %zu workspace bytes, got %zu",
                        need, workspace ? workspace_bytes : (size_t)0);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(MLXQ_ERR_ALIGN, "quantized_matmul: workspace must be 256-byte aligned");
    }
    mlxq::QmvParams p{};
    p.x = x; p.w = w; p.s = scales; p.b = biases; p.bias = bias; p.out = out;
    p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
    p.mode = 0; p.lhs = nullptr; p.lhs_div = 1; p.rhs = nullptr; p.seg = nullptr;
    p.batch = 0; p.num_experts = 1; p.x_batches = 1; p.w_estride = 0; p.sb_estride = 0;
    p.splits = plan.splits; p.gps = plan.gps; p.win = plan.win; p.ztotal = plan.ztotal;
    if (need > 0) {
        p.counter = static_cast<unsigned*>(workspace);
        p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + mlxq::kTicketBytes);
    }
    plan.overlap = mlxq::launch_overlap_enabled();
    cudaError_t e = mlxq::qmv_launch(dtype, bits, group_size, plan, p,
                                     static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul launch");
    return MLXQ_OK;
}

int mlxq_swiglu_supported(int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype) {
    if (check_bits_gs(bits, group_size, true) || check_k(K, group_size)) return 0;
    if (M <= 0 || N <= 0 || N % 16 || M > kIntMax || N > kIntMax || K > kIntMax) return 0;
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16) return 0;
    DeviceInfo di;
    if (device_info(&di, nullptr)) return 0;
    if (mlxq::qgemm_supported(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), bits,
                              group_size))
        return 1;
    mlxq::QtPlan tplan;
    return mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                              static_cast<int>(K), di.num_sms, di.max_smem, di.sm_smem, &tplan)
               ? 1 : 0;
}

int mlxq_quantized_matmul_swiglu(const void* x, const uint32_t* w, const void* scales,
                                 const void* biases, void* out, int64_t M, int64_t N, int64_t K,
                                 int group_size, int bits, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    int rc = check_bits_gs(bits, group_size, true);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (M < 0 || N <= 0 || N % 16 || M > kIntMax || N > kIntMax || K > kIntMax)
        return fail(MLXQ_ERR_SHAPE,
                    "quantized_matmul_swiglu: bad shape M=%lld N=%lld K=%lld (N: gate + up rows, "
                    "a multiple of 16)", (long long)M, (long long)N, (long long)K);
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "quantized_matmul_swiglu: dtype must be bfloat16 or float16");
    if (!x || !w || !scales || !biases || !out)
        return fail(MLXQ_ERR_NULL, "quantized_matmul_swiglu: NULL pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases) ||
        !aligned16(out))
        return fail(MLXQ_ERR_ALIGN, "quantized_matmul_swiglu: pointers must be 16-byte aligned");
    if (M == 0) return MLXQ_OK;
    DeviceInfo di;
    if ((rc = device_info(&di, static_cast<cudaStream_t>(stream)))) return rc;
    if (mlxq::qgemm_supported(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), bits,
                              group_size)) {
        // prefill: the tcgen05 kernel's whole tiles with the SwiGLU epilogue
        mlxq::QgemmParams q{};
        q.x = x; q.w = w; q.s = scales; q.b = biases; q.bias = nullptr; q.out = out;
        q.M = static_cast<int>(M); q.N = static_cast<int>(N); q.K = static_cast<int>(K);
        q.epi = 1;
        cudaError_t e = mlxq::qgemm_launch(dtype, bits, group_size, q,
                                           static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul_swiglu (prefill) launch");
        return MLXQ_OK;
    }
    mlxq::QtPlan tplan;
    if (!mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                            static_cast<int>(K), di.num_sms, di.max_smem, di.sm_smem, &tplan))
        return fail(MLXQ_ERR_SHAPE,
                    "quantized_matmul_swiglu: no plan (decode kernel: M <= 16, K/group_size a "
                    "multiple of 8; prefill kernel: M > 32, K a multiple of 64); see "
                    "mlxq_swiglu_supported");
    if (tplan.ws_bytes > 0) {
        if (!workspace || workspace_bytes < tplan.ws_bytes)
            return fail(MLXQ_ERR_WORKSPACE,
                        "quantized_matmul_swiglu: needs %zu workspace bytes, got %zu",
                        tplan.ws_bytes, workspace ? workspace_bytes : (size_t)0);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(MLXQ_ERR_ALIGN, "quantized_matmul_swiglu: workspace must be 256-byte aligned");
    }
    cudaError_t e = mlxq::qmv_tma_launch(
        dtype, bits, group_size, tplan, x, w, scales, biases, nullptr, out, static_cast<int>(M),
        static_cast<int>(N), static_cast<int>(K), workspace, mlxq::launch_overlap_enabled(),
        static_cast<cudaStream_t>(stream), 1);
    if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul_swiglu launch");
    return MLXQ_OK;
}

size_t mlxq_argmax_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                  int dtype) {
    if (check_bits_gs(bits, group_size, true) || check_k(K, group_size)) return 0;
    if (M <= 0 || N <= 0 || M > kIntMax || N > kIntMax || K > kIntMax) return 0;
    DeviceInfo di;
    if (device_info(&di, nullptr)) return 0;
    mlxq::QtPlan tplan;
    if (!mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                            static_cast<int>(K), di.num_sms, di.max_smem, di.sm_smem, &tplan))
        return 0;
    return tplan.ws_bytes > mlxq::kTicketBytes ? tplan.ws_bytes : mlxq::kTicketBytes;
}

int mlxq_quantized_matmul_argmax(const void* x, const uint32_t* w, const void* scales,
                                 const void* biases, const void* bias, int32_t* ids, int64_t M,
                                 int64_t N, int64_t K, int group_size, int bits, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_bits_gs(bits, group_size, true);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (M < 0 || N <= 0 || M > kIntMax || N > kIntMax || K > kIntMax)
        return fail(MLXQ_ERR_SHAPE, "quantized_matmul_argmax: bad shape M=%lld N=%lld K=%lld",
                    (long long)M, (long long)N, (long long)K);
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "quantized_matmul_argmax: dtype must be bfloat16 or float16");
    if (!x || !w || !scales || !biases || !ids)
        return fail(MLXQ_ERR_NULL, "quantized_matmul_argmax: NULL pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases) ||
        (bias && !aligned16(bias)))
        return fail(MLXQ_ERR_ALIGN, "quantized_matmul_argmax: pointers must be 16-byte aligned");
    if (M == 0) return MLXQ_OK;
    DeviceInfo di;
    if ((rc = device_info(&di, static_cast<cudaStream_t>(stream)))) return rc;
    mlxq::QtPlan tplan;
    if (!mlxq::qmv_tma_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                            static_cast<int>(K), di.num_sms, di.max_smem, di.sm_smem, &tplan))
        return fail(MLXQ_ERR_SHAPE,
                    "quantized_matmul_argmax: decode shapes only (M <= 16, K/group_size a "
                    "multiple of 8)");
    const size_t need = tplan.ws_bytes > mlxq::kTicketBytes ? tplan.ws_bytes : mlxq::kTicketBytes;
    if (!workspace || workspace_bytes < need)
        return fail(MLXQ_ERR_WORKSPACE, "quantized_matmul_argmax: needs %zu workspace bytes, got %zu",
                    need, workspace ? workspace_bytes : (size_t)0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u)
        return fail(MLXQ_ERR_ALIGN, "quantized_matmul_argmax: workspace must be 256-byte aligned");
    cudaError_t e = mlxq::qmv_tma_launch(
        dtype, bits, group_size, tplan, x, w, scales, biases, bias, ids, static_cast<int>(M),
        static_cast<int>(N), static_cast<int>(K), workspace, mlxq::launch_overlap_enabled(),
        static_cast<cudaStream_t>(stream), 2);
    if (e != cudaSuccess) return cuda_fail(e, "quantized_matmul_argmax launch");
    return MLXQ_OK;
}

size_t mlxq_gather_qmm_workspace_size(int64_t batch, int64_t M, int64_t N, int64_t K,
                                      int64_t num_experts, int group_size, int bits, int dtype,
                                      int sorted_indices) {
    (void)batch; (void)M; (void)N; (void)K; (void)group_size; (void)bits; (void)dtype;
    if (!sorted_indices || num_experts <= 0) return 0;
    // expert segment table [E+1], then the grouped kernel's tile offsets [E+1]
    return (2 * (static_cast<size_t>(num_experts) + 1) * 4 + 255) / 256 * 256;
}

// MLXQ_GATHER_KERNEL=cpasync (read once per process) sends decode-sized gather_qmm
// calls to the cp.async kernel instead of the TMA-fed grouped one.
static bool gather_cpasync_forced() {
    static const bool v = [] {
        const char* e = std::getenv("MLXQ_GATHER_KERNEL");
        return e && std::strcmp(e, "cpasync") == 0;
    }();
    return v;
}

// Argument checks shared by the gather_qmm entry points (`what` names the caller).
static int check_gather(const char* what, const void* x, const uint32_t* w, const void* scales,
                        const void* biases, const int32_t* lhs_indices, int64_t lhs_div,
                        const int32_t* rhs_indices, const void* out, int64_t batch, int64_t M,
                        int64_t N, int64_t K, int64_t num_experts, int64_t x_batches,
                        int group_size, int bits, int dtype) {
    int rc = check_bits_gs(bits, group_size, true);
    if (rc) return rc;
    if ((rc = check_k(K, group_size))) return rc;
    if (batch < 0 || M < 0 || N <= 0 || num_experts <= 0 || x_batches <= 0 || batch > kIntMax ||
        M > kIntMax || N > kIntMax || K > kIntMax || num_experts > kIntMax ||
        x_batches > kIntMax || batch * M > kIntMax || x_batches * M > kIntMax)
        return fail(MLXQ_ERR_SHAPE,
                    "%s: bad shape batch=%lld M=%lld N=%lld K=%lld E=%lld x_batches=%lld", what,
                    (long long)batch, (long long)M, (long long)N, (long long)K,
                    (long long)num_experts, (long long)x_batches);
    if (!lhs_indices && lhs_div < 1)
        return fail(MLXQ_ERR_INDEX, "%s: lhs_div must be >= 1 without lhs_indices", what);
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16)
        return fail(MLXQ_ERR_DTYPE, "%s: dtype=%d must be bfloat16 or float16", what, dtype);
    if (!x || !w || !scales || !biases || !out || !rhs_indices)
        return fail(MLXQ_ERR_NULL, "%s: NULL pointer", what);
    if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases) ||
        !aligned16(out))
        return fail(MLXQ_ERR_ALIGN, "%s: pointers must be 16-byte aligned", what);
    return MLXQ_OK;
}

// Sorted rows (no lhs, one x row block per entry) with enough rows per expert for the
// grouped tcgen05 GEMM.
static bool grouped_prefill_applies(bool lhs_given, int64_t lhs_div, int64_t batch, int64_t M,
                                    int64_t N, int64_t K, int64_t num_experts, int64_t x_batches,
                                    int group_size, int bits, int sorted_indices) {
    return sorted_indices && !lhs_given && lhs_div == 1 && x_batches == batch &&
           batch * M >= kGroupedMinRows * num_experts &&
           mlxq::qgemm_supported(static_cast<int>(batch * M), static_cast<int>(N),
                                 static_cast<int>(K), bits, group_size);
}

// The grouped decode plan for a gather_qmm call; false when its kernel does not take
// the shape (or MLXQ_GATHER_KERNEL=cpasync asks for the cp.async kernel).
static bool gather_decode_plan(const DeviceInfo& di, bool lhs_given, int64_t lhs_div,
                               int64_t batch, int64_t M, int64_t N, int64_t K,
                               int64_t num_experts, int64_t x_batches, int group_size, int bits,
                               int sorted_indices, mlxq::QgdPlan* plan) {
    if (gather_cpasync_forced()) return false;
    const bool rows_sorted = sorted_indices && !lhs_given && lhs_div == 1 && x_batches == batch;
    // enough rows per expert for the grouped tcgen05 GEMM (mlxq_gather_qmm takes it first)
    if (grouped_prefill_applies(lhs_given, lhs_div, batch, M, N, K, num_experts, x_batches,
                                group_size, bits, sorted_indices))
        return false;
    return mlxq::qmv_grouped_plan(bits, group_size, batch, static_cast<int>(M),
                                  static_cast<int>(N), static_cast<int>(K),
                                  static_cast<int>(num_experts), rows_sorted, di.num_sms,
                                  di.max_smem, di.sm_smem, plan);
}

// The grouped tcgen05 GEMM: the segment table and per-expert tile offsets in the
// workspace (mlxq_gather_qmm_workspace_size), then the kernel (epi 1: SwiGLU epilogue).
static int launch_grouped_prefill(const void* x, const uint32_t* w, const void* scales,
                                  const void* biases, void* out, const int32_t* rhs_indices,
                                  int64_t batch, int64_t M, int64_t N, int64_t K,
                                  int64_t num_experts, int group_size, int bits, int dtype,
                                  void* workspace, cudaStream_t st, int epi) {
    int32_t* seg = static_cast<int32_t*>(workspace);
    int32_t* tile_start = seg + (num_experts + 1);
    cudaError_t e = mlxq::launch_segments(rhs_indices, static_cast<int>(batch),
                                          static_cast<int>(num_experts), seg, st);
    if (e == cudaSuccess)
        e = mlxq::launch_group_tiles(seg, static_cast<int>(num_experts), static_cast<int>(M),
                                     static_cast<int>(N), tile_start, st);
    if (e != cudaSuccess) return cuda_fail(e, "gather_qmm segment table");
    mlxq::QgemmParams q{};
    q.x = x; q.w = w; q.s = scales; q.b = biases; q.bias = nullptr; q.out = out;
    q.M = static_cast<int>(batch * M); q.N = static_cast<int>(N); q.K = static_cast<int>(K);
    q.E = static_cast<int>(num_experts); q.rpe = static_cast<int>(M);
    q.seg = seg; q.tile_start = tile_start;
    q.epi = epi;
    e = mlxq::qgemm_launch(dtype, bits, group_size, q, st);
    if (e != cudaSuccess) return cuda_fail(e, "gather_qmm (grouped) launch");
    return MLXQ_OK;
}

int mlxq_gather_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases,
                    const int32_t* lhs_indices, int64_t lhs_div, const int32_t* rhs_indices,
                    void* out, int64_t batch, int64_t M, int64_t N, int64_t K,
                    int64_t num_experts, int64_t x_batches, int group_size, int bits, int dtype,
                    int sorted_indices, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_gather("gather_qmm", x, w, scales, biases, lhs_indices, lhs_div, rhs_indices,
                          out, batch, M, N, K, num_experts, x_batches, group_size, bits, dtype);
    if (rc) return rc;
    if (batch == 0 || M == 0) return MLXQ_OK;
    DeviceInfo di;
    if ((rc = device_info(&di, static_cast<cudaStream_t>(stream)))) return rc;
    const int mode = sorted_indices ? 2 : 1;
    const size_t need = mlxq_gather_qmm_workspace_size(batch, M, N, K, num_experts, group_size,
                                                       bits, dtype, sorted_indices);
    if (need > 0) {
        if (!workspace || workspace_bytes < need)
            return fail(MLXQ_ERR_WORKSPACE, "gather_qmm: needs %zu workspace bytes, got %zu", need,
                        workspace ? workspace_bytes : (size_t)0);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(MLXQ_ERR_ALIGN, "gather_qmm: workspace must be 256-byte aligned");
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Sorted, one x row block per entry, enough rows per expert: grouped tcgen05 GEMM
    // over the experts' contiguous row segments.
    if (grouped_prefill_applies(lhs_indices != nullptr, lhs_div, batch, M, N, K, num_experts,
                                x_batches, group_size, bits, sorted_indices)) {
        rc = launch_grouped_prefill(x, w, scales, biases, out, rhs_indices, batch, M, N, K,
                                    num_experts, group_size, bits, dtype, workspace, st, 0);
        return rc;
    }
    // Otherwise the TMA-fed grouped decode kernel: sorted rows of an expert taken
    // together, else one entry at a time (the cp.async kernel below when its plan does
    // not fit, or when MLXQ_GATHER_KERNEL=cpasync asks for it, for comparisons).
    {
        mlxq::QgdPlan gp;
        if (gather_decode_plan(di, lhs_indices != nullptr, lhs_div, batch, M, N, K, num_experts, x_batches,
                               group_size, bits, sorted_indices, &gp)) {
            cudaError_t e = mlxq::qmv_grouped_launch(
                dtype, bits, group_size, gp, x, w, scales, biases, out, rhs_indices, lhs_indices,
                static_cast<int>(lhs_div < 1 ? 1 : lhs_div), static_cast<int>(batch),
                static_cast<int>(x_batches), static_cast<int>(M), static_cast<int>(N),
                static_cast<int>(K), static_cast<int>(num_experts),
                mlxq::launch_overlap_enabled(), st);
            if (e != cudaSuccess) return cuda_fail(e, "gather_qmm (grouped decode) launch");
            return MLXQ_OK;
        }
    }
    mlxq::QmvPlan plan;
    const int zhint = (mode == 2) ? static_cast<int>(batch * M / num_experts) : static_cast<int>(batch);
    if (!mlxq::qmv_plan(dtype, bits, group_size, static_cast<int>(M), static_cast<int>(N),
                        static_cast<int>(K), mode, zhint, di.num_sms, di.max_smem, &plan))
        return fail(MLXQ_ERR_SHAPE, "gather_qmm: no launch plan fits shared memory");
    if (mode == 2) {
        plan.ztotal = static_cast<int>(num_experts);
        plan.gridz = plan.ztotal < 65535 ? plan.ztotal : 65535;
    }
    mlxq::QmvParams p{};
    p.x = x; p.w = w; p.s = scales; p.b = biases; p.bias = nullptr; p.out = out;
    p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
    p.mode = mode; p.lhs = lhs_indices; p.lhs_div = static_cast<int>(lhs_div < 1 ? 1 : lhs_div);
    p.rhs = rhs_indices; p.batch = static_cast<int>(batch);
    p.num_experts = static_cast<int>(num_experts); p.x_batches = static_cast<int>(x_batches);
    p.w_estride = N * (K * bits / 32);
    p.sb_estride = N * (K / group_size);
    p.splits = 1; p.gps = plan.gps; p.win = plan.win; p.ztotal = plan.ztotal;
    p.partial = nullptr; p.counter = nullptr;
    if (mode == 2) {
        int32_t* seg = static_cast<int32_t*>(workspace);
        cudaError_t e = mlxq::launch_segments(rhs_indices, static_cast<int>(batch),
                                              static_cast<int>(num_experts), seg, st);
        if (e != cudaSuccess) return cuda_fail(e, "gather_qmm segment table");
        p.seg = seg;
    }
    plan.overlap = false;  // index arrays come from the kernels just before
    cudaError_t e = mlxq::qmv_launch(dtype, bits, group_size, plan, p, st);
    if (e != cudaSuccess) return cuda_fail(e, "gather_qmm launch");
    return MLXQ_OK;
}

int mlxq_gather_swiglu_supported(int64_t batch, int64_t M, int64_t N, int64_t K,
                                 int64_t num_experts, int64_t x_batches, int group_size, int bits,
                                 int dtype, int lhs_given, int sorted_indices) {
    if (check_bits_gs(bits, group_size, true) || check_k(K, group_size)) return 0;
    if (dtype != MLXQ_BF16 && dtype != MLXQ_F16) return 0;
    if (batch < 1 || M < 1 || N < 16 || N % 16 || num_experts < 1 || x_batches < 1 ||
        batch > kIntMax || M > kIntMax || N > kIntMax || K > kIntMax ||
        num_experts > kIntMax || x_batches > kIntMax || batch * M > kIntMax ||
        x_batches * M > kIntMax)
        return 0;
    if (grouped_prefill_applies(lhs_given != 0, 1, batch, M, N, K, num_experts, x_batches,
                                group_size, bits, sorted_indices))
        return 1;
    DeviceInfo di;
    if (device_info(&di, nullptr)) return 0;
    mlxq::QgdPlan gp;
    return gather_decode_plan(di, lhs_given != 0, 1, batch, M, N, K, num_experts, x_batches,
                              group_size, bits, sorted_indices, &gp) ? 1 : 0;
}

int mlxq_gather_qmm_swiglu(const void* x, const uint32_t* w, const void* scales,
                           const void* biases, const int32_t* lhs_indices, int64_t lhs_div,
                           const int32_t* rhs_indices, void* out, int64_t batch, int64_t M,
                           int64_t N, int64_t K, int64_t num_experts, int64_t x_batches,
                           int group_size, int bits, int dtype, int sorted_indices,
                           void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_gather("gather_qmm_swiglu", x, w, scales, biases, lhs_indices, lhs_div,
                          rhs_indices, out, batch, M, N, K, num_experts, x_batches, group_size,
                          bits, dtype);
    if (rc) return rc;
    if (N % 16)
        return fail(MLXQ_ERR_SHAPE, "gather_qmm_swiglu: N=%lld must hold 16-row gate/up tiles",
                    (long long)N);
    if (batch == 0 || M == 0) return MLXQ_OK;
    DeviceInfo di;
    if ((rc = device_info(&di, static_cast<cudaStream_t>(stream)))) return rc;
    if (grouped_prefill_applies(lhs_indices != nullptr, lhs_div, batch, M, N, K, num_experts,
                                x_batches, group_size, bits, sorted_indices)) {
        const size_t need = mlxq_gather_qmm_workspace_size(batch, M, N, K, num_experts,
                                                           group_size, bits, dtype, 1);
        if (!workspace || workspace_bytes < need)
            return fail(MLXQ_ERR_WORKSPACE, "gather_qmm_swiglu: needs %zu workspace bytes, got %zu",
                        need, workspace ? workspace_bytes : (size_t)0);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(MLXQ_ERR_ALIGN, "gather_qmm_swiglu: workspace must be 256-byte aligned");
        return launch_grouped_prefill(x, w, scales, biases, out, rhs_indices, batch, M, N, K,
                                      num_experts, group_size, bits, dtype, workspace,
                                      static_cast<cudaStream_t>(stream), 1);
    }
    mlxq::QgdPlan gp;
    if (!gather_decode_plan(di, lhs_indices != nullptr, lhs_div, batch, M, N, K, num_experts,
                            x_batches, group_size, bits, sorted_indices, &gp))
        return fail(MLXQ_ERR_SHAPE,
                    "gather_qmm_swiglu: no plan for this shape (call gather_qmm and apply the "
                    "activation)");
    cudaError_t e = mlxq::qmv_grouped_launch(
        dtype, bits, group_size, gp, x, w, scales, biases, out, rhs_indices, lhs_indices,
        static_cast<int>(lhs_div < 1 ? 1 : lhs_div), static_cast<int>(batch),
        static_cast<int>(x_batches), static_cast<int>(M), static_cast<int>(N),
        static_cast<int>(K), static_cast<int>(num_experts), mlxq::launch_overlap_enabled(),
        static_cast<cudaStream_t>(stream), 1);
    if (e != cudaSuccess) return cuda_fail(e, "gather_qmm_swiglu launch");
    return MLXQ_OK;
}

}  // extern "C"
