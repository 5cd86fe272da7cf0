/*
 * qmm_oracle.c -- CPU restatement of MLX's group-wise affine quantization
 * family (quantize / dequantize / quantized_matmul / gather_qmm).
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library in mlx-server-runtime_b200/csrc. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it; the product path never does.
 *
 * Parity status: UNPINNED against the reference. The arithmetic lives in the
 * third-party package mlx 0.31.2 (pinned in the reference at
 * python/uv.lock:939-940); its source is not vendored under the reference tree,
 * it cannot be installed in this environment, and the reference's own tests
 * construct no quantized layer (no golden vectors exist). This restatement
 * follows MLX's published CPU algorithm as documented for mlx.core.quantize /
 * dequantize / quantized_matmul / gather_qmm, cross-checked against an
 * independent numpy restatement (oracle/oracle_np.py) and hand-derived
 * known-answer vectors (tests/golden/).
 *
 * Call sites it stands in for (reference tree):
 *   mx.quantize            python/mlx_worker/native_mlx/models/lfm2.py:112-117,142-151
 *   nn.quantize            python/mlx_worker/native_mlx/models/qwen2.py:318-324
 *   QuantizedLinear (qmm)  python/mlx_worker/native_mlx/models/qwen2.py:58-61,123-134
 *   mx.gather_qmm          python/mlx_worker/native_mlx/models/lfm2.py:176-187
 *
 * Storage layout (MLX "affine" mode):
 *   w_q     uint32 [rows, K*bits/32]; code k of a row sits in word k/(32/bits)
 *           at bits [bits*(k%(32/bits)), +bits) -- lowest K index in the
 *           least-significant bits.
 *   scales  [rows, K/group_size], dtype of the unquantized weight
 *   biases  [rows, K/group_size], same dtype;  w ~= scale*q + bias
 *
 * dtype codes: 0 = float32, 1 = bfloat16, 2 = float16 (same as include/mlxq_b200.h)
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off, so that no
 * multiply-add is fused and every rounding step below is explicit).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OQ_F32 = 0, OQ_BF16 = 1, OQ_F16 = 2 };

/* ---- scalar conversions (round to nearest even) --------------------------- */
static inline float bf16_to_f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float f16_to_f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}
static inline uint16_t f_to_f16(float f) {
    _Float16 v = (_Float16)f; /* IEEE round-to-nearest-even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
static inline float ld(const void* p, int dt, size_t i) {
    if (dt == OQ_F32) return ((const float*)p)[i];
    if (dt == OQ_BF16) return bf16_to_f(((const uint16_t*)p)[i]);
    return f16_to_f(((const uint16_t*)p)[i]);
}
/* round a float to the storage precision of dtype dt (and back) */
static inline float rnd(float f, int dt) {
    if (dt == OQ_F32) return f;
    if (dt == OQ_BF16) return bf16_to_f(f_to_bf16(f));
    return f16_to_f(f_to_f16(f));
}
static inline void st(void* p, int dt, size_t i, float f) {
    if (dt == OQ_F32) ((float*)p)[i] = f;
    else if (dt == OQ_BF16) ((uint16_t*)p)[i] = f_to_bf16(f);
    else ((uint16_t*)p)[i] = f_to_f16(f);
}

static int check_common(int64_t K, int group_size, int bits) {
    if (bits != 2 && bits != 4 && bits != 8) return -4;
    if (group_size != 32 && group_size != 64 && group_size != 128) return -5;
    if (K <= 0 || K % group_size) return -1;
    return 0;
}

/*
 * quantize: per group of `group_size` consecutive elements of a row
 * (MLX affine quantizer):
 *   w_max, w_min over the group (in float)
 *   mask  = |w_min| > |w_max|
 *   scale = max((w_max - w_min) / (2^bits - 1), 1e-7), negated when !mask
 *   edge  = mask ? w_min : w_max
 *   q0    = rint(edge / scale)
 *   if q0 != 0: scale = edge / q0, bias = edge      (the larger-magnitude
 *   else:       bias = 0                             endpoint is exact)
 *   code  = clamp(rint((w - bias) / scale), 0, 2^bits - 1)
 *   scale, bias stored in w's dtype (round to nearest even).
 * The codes use the float scale/bias, before they are rounded for storage.
 */
int oq_quantize(const void* w, int dt, uint32_t* wq, void* scales, void* biases,
                int64_t rows, int64_t K, int group_size, int bits) {
    int rc = check_common(K, group_size, bits);
    if (rc) return rc;
    const int64_t G = K / group_size;
    const int epw = 32 / bits;
    const float n_bins = (float)((1 << bits) - 1);
    const float eps = 1e-7f;
#pragma omp parallel for schedule(static)
    for (int64_t gi = 0; gi < rows * G; ++gi) {
        const size_t base = (size_t)gi * group_size;
        float w_max = -INFINITY, w_min = INFINITY;
        for (int j = 0; j < group_size; ++j) {
            float v = ld(w, dt, base + j);
            w_max = v > w_max ? v : w_max;
            w_min = v < w_min ? v : w_min;
        }
        int mask = fabsf(w_min) > fabsf(w_max);
        float scale = (w_max - w_min) / n_bins;
        scale = scale > eps ? scale : eps;
        scale = mask ? scale : -scale;
        float edge = mask ? w_min : w_max;
        float q0 = rintf(edge / scale);
        float bias = 0.0f;
        if (q0 != 0.0f) {
            scale = edge / q0;
            bias = edge;
        }
        uint32_t* out = wq + (size_t)gi * (group_size / epw);
        for (int j = 0; j < group_size / epw; ++j) {
            uint32_t word = 0;
            for (int e = 0; e < epw; ++e) {
                float v = ld(w, dt, base + (size_t)j * epw + e);
                float q = rintf((v - bias) / scale);
                q = q < 0.0f ? 0.0f : q;
                q = q > n_bins ? n_bins : q;
                word |= (uint32_t)q << (bits * e);
            }
            out[j] = word;
        }
        st(scales, dt, (size_t)gi, scale);
        st(biases, dt, (size_t)gi, bias);
    }
    return 0;
}

/*
 * dequantize: out = scale * q + bias evaluated in the storage dtype one
 * operation at a time, as MLX's CPU path does with its bf16/fp16 scalar
 * types: t = round(scale * q); out = round(t + bias).
 */
int oq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int dt,
                  void* out, int64_t rows, int64_t K, int group_size, int bits) {
    int rc = check_common(K, group_size, bits);
    if (rc) return rc;
    const int epw = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t words = rows * K / epw;
#pragma omp parallel for schedule(static)
    for (int64_t wi = 0; wi < words; ++wi) {
        const size_t g = (size_t)(wi * epw / group_size);
        const float s = ld(scales, dt, g), b = ld(biases, dt, g);
        uint32_t word = wq[wi];
        for (int e = 0; e < epw; ++e) {
            float q = (float)((word >> (bits * e)) & mask);
            float t = rnd(s * q, dt);
            st(out, dt, (size_t)wi * epw + e, t + b);
        }
    }
    return 0;
}

/* one output row-vector: acc over K of x[k] * (s*q + b) in float */
static void qdot_row(const void* x, int dt, const uint32_t* wrow, const void* scales,
                     const void* biases, size_t sb_off, int64_t K, int group_size,
                     int bits, float* acc_out) {
    const int epw = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    float acc = 0.0f;
    for (int64_t g = 0; g < K / group_size; ++g) {
        const float s = ld(scales, dt, sb_off + g), b = ld(biases, dt, sb_off + g);
        for (int j = 0; j < group_size; ++j) {
            const int64_t k = g * group_size + j;
            const uint32_t word = wrow[k / epw];
            const float q = (float)((word >> (bits * (k % epw))) & mask);
            const float wv = s * q + b;
            acc += ld(x, dt, (size_t)k) * wv;
        }
    }
    *acc_out = acc;
}

/*
 * quantized_matmul(x, w, scales, biases, transpose=True): out[m, n] =
 * round(sum_k x[m,k] * (scale[n,k/g]*q[n,k] + bias[n,k/g])), accumulated in
 * float32. An optional per-output `bias` vector (the Linear bias of Qwen2's
 * q/k/v projections) is added afterwards as a separate rounded add, as the
 * QuantizedLinear module does.
 */
int oq_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                        const void* biases, const void* bias, int dt, void* out,
                        int64_t M, int64_t N, int64_t K, int group_size, int bits) {
    int rc = check_common(K, group_size, bits);
    if (rc) return rc;
    if (dt != OQ_BF16 && dt != OQ_F16 && dt != OQ_F32) return -2;
    const int64_t kw = K * bits / 32, G = K / group_size;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float acc;
            const size_t xoff = (size_t)(m * K);
            const char* xb = (const char*)x + xoff * (dt == OQ_F32 ? 4 : 2);
            qdot_row(xb, dt, w + n * kw, scales, biases, (size_t)(n * G), K, group_size,
                     bits, &acc);
            float y = rnd(acc, dt);
            if (bias) y = rnd(y + ld(bias, dt, (size_t)n), dt);
            st(out, dt, (size_t)(m * N + n), y);
        }
    }
    return 0;
}

/*
 * gather_qmm: out[b] = x[xi(b)] @ dequant(w[rhs[b]])^T, with x viewed as
 * [x_batches, M, K], w as [E, N, K*bits/32], scales/biases as [E, N, K/g],
 * out as [batch, M, N]; xi(b) = lhs ? lhs[b] : b / lhs_div. `sorted_indices`
 * in MLX is a performance hint only and does not change results, so it is
 * not a parameter here.
 */
int oq_gather_qmm(const void* x, const uint32_t* w, const void* scales,
                  const void* biases, const int32_t* lhs, int64_t lhs_div,
                  const int32_t* rhs, int dt, void* out, int64_t batch, int64_t M,
                  int64_t N, int64_t K, int64_t E, int64_t x_batches, int group_size,
                  int bits) {
    int rc = check_common(K, group_size, bits);
    if (rc) return rc;
    const int64_t kw = K * bits / 32, G = K / group_size;
    const int esz = dt == OQ_F32 ? 4 : 2;
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t xi = lhs ? lhs[b] : b / (lhs_div > 0 ? lhs_div : 1);
        const int64_t e = rhs[b];
        if (xi < 0 || xi >= x_batches || e < 0 || e >= E) return -1;
    }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t n = 0; n < N; ++n) {
            const int64_t xi = lhs ? lhs[b] : b / (lhs_div > 0 ? lhs_div : 1);
            const int64_t e = rhs[b];
            for (int64_t m = 0; m < M; ++m) {
                float acc;
                const char* xr = (const char*)x + (size_t)((xi * M + m) * K) * esz;
                qdot_row(xr, dt, w + (e * N + n) * kw, scales, biases,
                         (size_t)((e * N + n) * G), K, group_size, bits, &acc);
                st(out, dt, (size_t)((b * M + m) * N + n), rnd(acc, dt));
            }
        }
    }
    return 0;
}

int oq_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oq_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
