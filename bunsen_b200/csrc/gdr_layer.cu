// The gated DeltaNet layer's steps around the rule (GatedDeltaNet::forward,
// crates/public/bunsen/src/blocks/transformers/mixers/gated_delta_net.rs:
// 396-440): the causal depthwise convolution with its silu and the q/k/v
// split, the gate production, the gated RMS norm of the rule's output, and
// the decode states' row reorder (linear_attention/state.rs:112-135). All of
// them are HBM-bound elementwise or row work on the CUDA cores: coalesced
// loads along the channel axis, f32 arithmetic, one pass over the data.
#include <cmath>
#include <type_traits>

#include "gdr_common.cuh"

namespace gdr {

// Device-side failures of this file's kernels since the last
// gdr_device_error: bit 1, a reorder source row outside the pool.
__device__ int g_layer_error;

cudaError_t take_layer_error(int* flag) {
    cudaError_t e = cudaMemcpyFromSymbol(flag, g_layer_error, sizeof(int));
    if (e != cudaSuccess || *flag == 0) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_layer_error, &zero, sizeof(int));
}

namespace {

// ---- causal depthwise convolution (causal_conv.rs:36-69) -------------------
struct Conv {
    int32_t n_seqs;
    int64_t tokens;             // all positions
    int32_t seq_len;            // dense: positions per sequence
    const int32_t* cu_seqlens;  // nullptr: dense
    int32_t channels, taps;     // C, K
    int32_t split0, split1;     // output channel cuts
    int32_t silu;
};

constexpr int kConvTokens = 64;    // positions per CTA
constexpr int kConvThreads = 128;  // channels per CTA, one per thread
constexpr int kMaxTaps = 8;

__device__ __forceinline__ void conv_span(const Conv& p, int s, int64_t& a, int64_t& b) {
    if (p.cu_seqlens == nullptr) {
        a = static_cast<int64_t>(s) * p.seq_len;
        b = a + p.seq_len;
        return;
    }
    a = p.cu_seqlens[s];
    b = p.cu_seqlens[s + 1];
    a = a < 0 ? 0 : (a > p.tokens ? p.tokens : a);
    b = b < a ? a : (b > p.tokens ? p.tokens : b);
}

// The sequence holding position t: the last s with start(s) <= t < end(s)
// (empty sequences skipped), by bisection over the offsets.
__device__ __forceinline__ int conv_seq_of(const Conv& p, int64_t t) {
    if (p.cu_seqlens == nullptr) return static_cast<int>(t / p.seq_len);
    int lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {  // first s with end(s) > t
        const int mid = (lo + hi) >> 1;
        int64_t a, b;
        conv_span(p, mid, a, b);
        if (b > t) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// One channel per thread, kConvTokens positions per CTA: each output needs
// only the K - 1 inputs before it, so windows run independently; the history
// at a window's (or a sequence's) start comes from x or from the state.
template <typename T, int K>
__global__ void __launch_bounds__(kConvThreads)
conv_kernel(const Conv p, const T* __restrict__ x, const T* __restrict__ weight,
            const float* state, T* out0, T* out1, T* out2) {
    const int c = blockIdx.x * kConvThreads + threadIdx.x;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kConvTokens;
    if (c >= p.channels || t0 >= p.tokens) return;
    const int C = p.channels;
    float w[K];
#pragma unroll
    for (int j = 0; j < K; ++j) w[j] = to_f32(weight[static_cast<int64_t>(c) * K + j]);
    int s = conv_seq_of(p, t0);
    int64_t start, end;
    conv_span(p, s, start, end);
    // The K - 1 inputs before t0, oldest first.
    float h[K - 1];
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
        const int64_t u = t0 - (K - 1) + i;
        h[i] = u >= start ? to_f32(x[u * C + c])
               : (state && start - u <= K - 1)
                   ? state[(static_cast<int64_t>(s) * (K - 1) + (K - 1) - (start - u)) * C + c]
                   : 0.f;
    }
    T* out;
    int64_t stride;
    int col;
    if (c < p.split0) {
        out = out0, stride = p.split0, col = c;
    } else if (c < p.split1) {
        out = out1, stride = p.split1 - p.split0, col = c - p.split0;
    } else {
        out = out2, stride = C - p.split1, col = c - p.split1;
    }
    const int64_t t1 = t0 + kConvTokens < p.tokens ? t0 + kConvTokens : p.tokens;
    for (int64_t t = t0; t < t1; ++t) {
        while (t >= end && s + 1 < p.n_seqs) {  // into the next sequence
            ++s;
            conv_span(p, s, start, end);
#pragma unroll
            for (int i = 0; i < K - 1; ++i)
                h[i] = state ? state[(static_cast<int64_t>(s) * (K - 1) + i) * C + c] : 0.f;
        }
        const float xt = to_f32(x[t * C + c]);
        float acc = h[0] * w[0];
#pragma unroll
        for (int j = 1; j < K - 1; ++j) acc = fmaf(h[j], w[j], acc);
        acc = fmaf(xt, w[K - 1], acc);
        if (p.silu) acc = silu(acc);
        out[t * stride + col] = from_f32<T>(acc);
#pragma unroll
        for (int i = 0; i + 1 < K - 1; ++i) h[i] = h[i + 1];
        h[K - 2] = xt;
    }
}

// Two adjacent channels per thread (4- or 8-byte accesses, a warp's row
// access one 128- or 256-byte line): few registers, so a full SM of warps
// keeps loads in flight while others compute; the positions of a window
// taken eight at a time, all eight rows loaded before any is used. Needs an
// even C, even splits and 8-byte-aligned buffers.
template <typename T>
__device__ __forceinline__ float2 load2(const T* p);
template <>
__device__ __forceinline__ float2 load2<float>(const float* p) {
    return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 load2<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <>
__device__ __forceinline__ float2 load2<__half>(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <typename T>
__device__ __forceinline__ void store2(T* p, float a, float b);
template <>
__device__ __forceinline__ void store2<float>(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <>
__device__ __forceinline__ void store2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
template <>
__device__ __forceinline__ void store2<__half>(__half* p, float a, float b) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
}

template <typename T, int K>
__global__ void __launch_bounds__(kConvThreads)
conv_vec_kernel(const Conv p, const T* __restrict__ x, const T* __restrict__ weight,
                const float* state, T* out0, T* out1, T* out2) {
    constexpr int kRows = 8;
    const int C = p.channels;
    const int c0 = (blockIdx.x * kConvThreads + threadIdx.x) * 2;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kConvTokens;
    if (c0 >= C || t0 >= p.tokens) return;
    float w0[K], w1[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        w0[j] = to_f32(weight[static_cast<int64_t>(c0) * K + j]);
        w1[j] = to_f32(weight[static_cast<int64_t>(c0 + 1) * K + j]);
    }
    auto from_state = [&](int s, int i) {
        return *reinterpret_cast<const float2*>(state + (static_cast<int64_t>(s) * (K - 1) + i) * C + c0);
    };
    int s = conv_seq_of(p, t0);
    int64_t start, end;
    conv_span(p, s, start, end);
    float2 h[K - 1];
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
        const int64_t u = t0 - (K - 1) + i;
        h[i] = u >= start ? load2(x + u * C + c0)
               : (state && start - u <= K - 1) ? from_state(s, static_cast<int>((K - 1) - (start - u)))
                                               : make_float2(0.f, 0.f);
    }
    T* out;
    int64_t stride;
    int col;
    if (c0 < p.split0) {
        out = out0, stride = p.split0, col = c0;
    } else if (c0 < p.split1) {
        out = out1, stride = p.split1 - p.split0, col = c0 - p.split0;
    } else {
        out = out2, stride = C - p.split1, col = c0 - p.split1;
    }
    const int64_t t1 = t0 + kConvTokens < p.tokens ? t0 + kConvTokens : p.tokens;
#pragma unroll 1
    for (int64_t tb = t0; tb < t1; tb += kRows) {
        float2 xr[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
            xr[r] = tb + r < t1 ? load2(x + (tb + r) * C + c0) : make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const int64_t t = tb + r;
            if (t < t1) {
                while (t >= end && s + 1 < p.n_seqs) {  // into the next sequence
                    ++s;
                    conv_span(p, s, start, end);
#pragma unroll
                    for (int i = 0; i < K - 1; ++i)
                        h[i] = state ? from_state(s, i) : make_float2(0.f, 0.f);
                }
                float a0 = h[0].x * w0[0], a1 = h[0].y * w1[0];
#pragma unroll
                for (int j = 1; j < K - 1; ++j) {
                    a0 = fmaf(h[j].x, w0[j], a0);
                    a1 = fmaf(h[j].y, w1[j], a1);
                }
                a0 = fmaf(xr[r].x, w0[K - 1], a0);
                a1 = fmaf(xr[r].y, w1[K - 1], a1);
                if (p.silu) {
                    a0 = silu(a0);
                    a1 = silu(a1);
                }
                store2(out + t * stride + col, a0, a1);
#pragma unroll
                for (int i = 0; i + 1 < K - 1; ++i) h[i] = h[i + 1];
                h[K - 2] = xr[r];
            }
        }
    }
}

// Two 16-bit values packed in a word, as f32 pairs.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// bf16 or f16 with C and the split points multiples of 8: a CTA walks kStageSpan
// positions of 1024 channels (eight per thread, one 16-byte load and store per
// position), the rows of each 16-position window staged into shared memory by
// cp.async while the window before is computed, so the loads stay in flight
// whatever the threads are doing (64 KiB per CTA). Positions run in stretches
// between sequence starts, so the per-position loop carries no boundary test
// and unrolls. The kernel is bound by instruction issue as much as by HBM: on
// B200, 131 072 positions x 8192 channels with silu run at 0.88 of the measured
// HBM copy rate this way (0.97 without silu; 0.57 with two channels per thread
// and a boundary test per position).
constexpr int kStageRows = 16, kStageCh = 8, kStageCols = kConvThreads * kStageCh,
              kStageSpan = 512;
constexpr uint32_t kStageBytes = 2u * kStageRows * kStageCols * 2;  // two windows

template <typename T, int K, bool kSilu>
__global__ void __launch_bounds__(kConvThreads, K <= 4 ? 4 : 2)
conv_staged_kernel(const Conv p, const T* __restrict__ x, const T* __restrict__ weight,
                   const float* state, T* out0, T* out1, T* out2) {
    constexpr int NP = kStageCh / 2;  // channel pairs per thread
    extern __shared__ __align__(16) uint8_t conv_smem[];
    auto* buf = reinterpret_cast<T*>(conv_smem);  // [2][16][1024]
    const int C = p.channels, tid = threadIdx.x;
    const int cb = blockIdx.x * kStageCols;
    const int c0 = cb + kStageCh * tid;
    const int64_t T0 = static_cast<int64_t>(blockIdx.y) * kStageSpan;
    if (T0 >= p.tokens) return;
    const int64_t T1 = T0 + kStageSpan < p.tokens ? T0 + kStageSpan : p.tokens;
    const int windows = static_cast<int>((T1 - T0 + kStageRows - 1) / kStageRows);
    auto load_window = [&](int w) {  // kStageRows rows x 128 16-byte pieces
        T* dst = buf + (w & 1) * kStageRows * kStageCols;
#pragma unroll 4
        for (int e = tid; e < kStageRows * (kStageCols / 8); e += kConvThreads) {
            const int r = e / (kStageCols / 8), piece = e % (kStageCols / 8);
            const int64_t t = T0 + static_cast<int64_t>(w) * kStageRows + r;
            const int c = cb + 8 * piece;
            const bool in = t < T1 && c < C;
            const T* src = x + (in ? t * C + c : 0);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(dst + r * kStageCols + 8 * piece))),
                         "l"(src), "r"(in ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_window(0);
    const bool active = c0 < C;
    float2 w[NP][K];      // the taps of channel pair q
    float2 h[NP][K - 1];  // the K - 1 inputs before the current position
    int s = 0;
    int64_t start = 0, end = 0;
    T* out = nullptr;
    int64_t stride = 0;
    int col = 0;
    if (active) {
#pragma unroll
        for (int q = 0; q < NP; ++q)
#pragma unroll
            for (int j = 0; j < K; ++j)
                w[q][j] = make_float2(to_f32(weight[static_cast<int64_t>(c0 + 2 * q) * K + j]),
                                      to_f32(weight[static_cast<int64_t>(c0 + 2 * q + 1) * K + j]));
        s = conv_seq_of(p, T0);
        conv_span(p, s, start, end);
#pragma unroll
        for (int i = 0; i < K - 1; ++i) {
            const int64_t u = T0 - (K - 1) + i;
#pragma unroll
            for (int q = 0; q < NP; ++q)
                h[q][i] = u >= start ? load2(x + u * C + c0 + 2 * q)
                          : (state && start - u <= K - 1)
                              ? *reinterpret_cast<const float2*>(
                                    state + (static_cast<int64_t>(s) * (K - 1) + (K - 1) - (start - u)) * C +
                                    c0 + 2 * q)
                              : make_float2(0.f, 0.f);
        }
        if (c0 < p.split0) {
            out = out0, stride = p.split0, col = c0;
        } else if (c0 < p.split1) {
            out = out1, stride = p.split1 - p.split0, col = c0 - p.split0;
        } else {
            out = out2, stride = C - p.split1, col = c0 - p.split1;
        }
    }
#pragma unroll 1
    for (int wi = 0; wi < windows; ++wi) {
        if (wi + 1 < windows) {
            load_window(wi + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // window wi has landed for every thread
        if (active) {
            const T* rows = buf + (wi & 1) * kStageRows * kStageCols + kStageCh * tid;
            const int64_t tw = T0 + static_cast<int64_t>(wi) * kStageRows;
            const int n = static_cast<int>(T1 - tw < kStageRows ? T1 - tw : kStageRows);
            int r = 0;
            while (r < n) {
                while (tw + r >= end && s + 1 < p.n_seqs) {  // into the next sequence
                    ++s;
                    conv_span(p, s, start, end);
#pragma unroll
                    for (int i = 0; i < K - 1; ++i)
#pragma unroll
                        for (int q = 0; q < NP; ++q)
                            h[q][i] = state ? *reinterpret_cast<const float2*>(
                                                  state + (static_cast<int64_t>(s) * (K - 1) + i) * C +
                                                  c0 + 2 * q)
                                            : make_float2(0.f, 0.f);
                }
                // Positions up to the next sequence start (the last sequence
                // runs to the window's end).
                const int stop = s + 1 < p.n_seqs && end - tw < n ? static_cast<int>(end - tw) : n;
#pragma unroll 3  // K = 4: the K - 1 history registers rotate in place
                for (; r < stop; ++r) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(rows + r * kStageCols);
                    const uint32_t xw[NP] = {xv.x, xv.y, xv.z, xv.w};
                    uint32_t y[NP];
#pragma unroll
                    for (int q = 0; q < NP; ++q) {
                        const float2 xt = unpack2<T>(xw[q]);
                        float a0 = h[q][0].x * w[q][0].x, a1 = h[q][0].y * w[q][0].y;
#pragma unroll
                        for (int j = 1; j < K - 1; ++j) {
                            a0 = fmaf(h[q][j].x, w[q][j].x, a0);
                            a1 = fmaf(h[q][j].y, w[q][j].y, a1);
                        }
                        a0 = fmaf(xt.x, w[q][K - 1].x, a0);
                        a1 = fmaf(xt.y, w[q][K - 1].y, a1);
                        if (kSilu) {
                            a0 = silu(a0);
                            a1 = silu(a1);
                        }
                        y[q] = pack2<T>(a0, a1);
#pragma unroll
                        for (int i = 0; i + 1 < K - 1; ++i) h[q][i] = h[q][i + 1];
                        h[q][K - 2] = xt;
                    }
                    *reinterpret_cast<uint4*>(out + (tw + r) * stride + col) =
                        make_uint4(y[0], y[1], y[2], y[3]);
                }
            }
        }
        __syncthreads();  // window wi's buffer is free for window wi + 2
    }
}

// The next state, per (sequence, channel): the last K - 1 inputs of the
// window [state, x], read in full before it is written (the state may be
// updated in place).
template <typename T>
__global__ void conv_state_kernel(const Conv p, const T* __restrict__ x, const float* state_in,
                                  float* state_out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int C = p.channels, K1 = p.taps - 1;
    if (i >= static_cast<int64_t>(p.n_seqs) * C) return;
    const int s = static_cast<int>(i / C), c = static_cast<int>(i % C);
    int64_t a, b;
    conv_span(p, s, a, b);
    const int64_t len = b - a;
    float old[kMaxTaps - 1];
#pragma unroll
    for (int j = 0; j < kMaxTaps - 1; ++j)
        old[j] = (j < K1 && state_in) ? state_in[(static_cast<int64_t>(s) * K1 + j) * C + c] : 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTaps - 1; ++j) {
        if (j >= K1) break;
        const int64_t pidx = len + j;  // index into [state (K - 1), x (len)]
        float v = 0.f;
        if (pidx < K1) {
#pragma unroll
            for (int m = 0; m < kMaxTaps - 1; ++m) v = (m == pidx) ? old[m] : v;
        } else {
            v = to_f32(x[(a + pidx - K1) * C + c]);
        }
        state_out[(static_cast<int64_t>(s) * K1 + j) * C + c] = v;
    }
}

// ---- gates (gated_delta_net.rs:422-426) ------------------------------------
template <typename T>
__global__ void gates_kernel(int64_t n, int heads, const T* __restrict__ a,
                             const T* __restrict__ b, const float* __restrict__ a_log,
                             const float* __restrict__ dt_bias, float* g, float* beta) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int h = static_cast<int>(i % heads);
        g[i] = gate_g(to_f32(a[i]), a_log[h], dt_bias[h]);
        beta[i] = gate_beta(to_f32(b[i]), std::is_same<T, __nv_bfloat16>::value ? GDR_DTYPE_BF16
                                          : std::is_same<T, __half>::value      ? GDR_DTYPE_F16
                                                                                 : GDR_DTYPE_F32);
    }
}

// ---- gated RMS norm (gated_delta_net.rs:439-440) ---------------------------
// One warp per (position, head) row of `width` features; `out` may be `x`.
template <typename T>
__global__ void gated_norm_kernel(int64_t rows, int width, const T* x, const T* __restrict__ z,
                                  const float* __restrict__ weight, float eps, T* out) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const T* xr = x + row * width;
    float ss = 0.f;
    for (int i = lane; i < width; i += 32) {
        const float v = to_f32(xr[i]);
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / width + eps);
    for (int i = lane; i < width; i += 32) {
        const float v = to_f32(xr[i]) * r * weight[i];
        out[row * width + i] = from_f32<T>(v * silu(to_f32(z[row * width + i])));
    }
}

// The bf16 or f16, 128-feature rows of the rule's output: 16 lanes per row, each 8
// features (16-byte accesses), so a warp instruction covers two rows; a warp
// takes kNormRows rows, every load issued before any is used. On B200,
// 4 Mi rows run at 1.03 of the measured HBM copy rate (0.82 with 8-byte
// accesses and 32 lanes per row; 8 or 16 rows per warp were slower).
constexpr int kNormRows = 4;
template <typename T>
__global__ void __launch_bounds__(256)
gated_norm_16b_128(int64_t rows, const T* x, const T* __restrict__ z,
                   const float* __restrict__ weight, float eps, T* out) {
    constexpr int kPairs = kNormRows / 2;
    const int lane = threadIdx.x & 31, half = lane >> 4, c = lane & 15;
    const int64_t r0 = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * kNormRows;
    if (r0 >= rows) return;
    const float4 w0 = reinterpret_cast<const float4*>(weight)[2 * c];
    const float4 w1 = reinterpret_cast<const float4*>(weight)[2 * c + 1];
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint4 xv[kPairs], zv[kPairs];
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
        int64_t row = r0 + 2 * i + half;
        row = row < rows ? row : r0;
        xv[i] = reinterpret_cast<const uint4*>(x + row * 128)[c];
        zv[i] = reinterpret_cast<const uint4*>(z + row * 128)[c];
    }
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
        const uint32_t xb[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        const uint32_t zb[4] = {zv[i].x, zv[i].y, zv[i].z, zv[i].w};
        float xf[8], ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t = unpack2<T>(xb[j]);
            xf[2 * j] = t.x;
            xf[2 * j + 1] = t.y;
            ss = fmaf(t.x, t.x, ss);
            ss = fmaf(t.y, t.y, ss);
        }
        // The 16 lanes of a row (the two halves of the warp reduce apart).
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss / 128.f + eps);
        const int64_t row = r0 + 2 * i + half;
        if (row < rows) {
            uint4 y;
            uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 zz = unpack2<T>(zb[j]);
                yw[j] = pack2<T>(xf[2 * j] * rs * wv[2 * j] * silu(zz.x),
                                 xf[2 * j + 1] * rs * wv[2 * j + 1] * silu(zz.y));
            }
            reinterpret_cast<uint4*>(out + row * 128)[c] = y;
        }
    }
}

// ---- state reorder (state.rs:112-135) --------------------------------------
// dst row r <- src row sources[r]; `words` 16-byte (or 4-byte) words per row.
template <typename W>
__global__ void reorder_kernel(const W* __restrict__ src, W* __restrict__ dst,
                               const int32_t* __restrict__ sources, int32_t rows,
                               int32_t src_rows, int64_t words) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < static_cast<int64_t>(rows) * words; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int32_t r = static_cast<int32_t>(i / words);
        const int64_t w = i % words;
        const int32_t from = sources[r];
        if (from < 0 || from >= src_rows) {
            if (w == 0) atomicOr(&g_layer_error, 2);
            continue;
        }
        dst[static_cast<int64_t>(r) * words + w] = src[static_cast<int64_t>(from) * words + w];
    }
}

int grid_for(int64_t n, int block) {
    const int64_t g = (n + block - 1) / block;
    return static_cast<int>(g < 148 * 16 ? (g > 0 ? g : 1) : 148 * 16);
}

template <typename T, int K>
void launch_conv_k(const Conv& p, const void* x, const void* w, const float* st, void* o0,
                   void* o1, void* o2, cudaStream_t s) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(st) |
                         reinterpret_cast<uintptr_t>(o0) | reinterpret_cast<uintptr_t>(o1) |
                         reinterpret_cast<uintptr_t>(o2);
    const bool vec = p.channels % 2 == 0 && p.split0 % 2 == 0 && p.split1 % 2 == 0 &&
                     (al & 7) == 0;
    const unsigned ty = static_cast<unsigned>((p.tokens + kConvTokens - 1) / kConvTokens);
    if constexpr (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value) {
        const uintptr_t al16 = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(o0) |
                               reinterpret_cast<uintptr_t>(o1) | reinterpret_cast<uintptr_t>(o2);
        if (vec && p.channels % kStageCh == 0 && p.split0 % kStageCh == 0 &&
            p.split1 % kStageCh == 0 && (al16 & 15) == 0) {
            auto* kern = p.silu ? conv_staged_kernel<T, K, true> : conv_staged_kernel<T, K, false>;
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kStageBytes));
            const dim3 grid((p.channels + kStageCols - 1) / kStageCols,
                            static_cast<unsigned>((p.tokens + kStageSpan - 1) / kStageSpan));
            kern<<<grid, kConvThreads, kStageBytes, s>>>(
                p, static_cast<const T*>(x), static_cast<const T*>(w), st, static_cast<T*>(o0),
                static_cast<T*>(o1), static_cast<T*>(o2));
            return;
        }
    }
    if (vec) {
        const dim3 grid((p.channels / 2 + kConvThreads - 1) / kConvThreads, ty);
        conv_vec_kernel<T, K><<<grid, kConvThreads, 0, s>>>(
            p, static_cast<const T*>(x), static_cast<const T*>(w), st, static_cast<T*>(o0),
            static_cast<T*>(o1), static_cast<T*>(o2));
        return;
    }
    const dim3 grid((p.channels + kConvThreads - 1) / kConvThreads, ty);
    conv_kernel<T, K><<<grid, kConvThreads, 0, s>>>(
        p, static_cast<const T*>(x), static_cast<const T*>(w), st, static_cast<T*>(o0),
        static_cast<T*>(o1), static_cast<T*>(o2));
}

template <typename T>
cudaError_t launch_conv_t(const Conv& p, const void* x, const void* w, const float* st_in,
                          void* o0, void* o1, void* o2, float* st_out, cudaStream_t s) {
    if (p.tokens > 0) {
        switch (p.taps) {
            case 2: launch_conv_k<T, 2>(p, x, w, st_in, o0, o1, o2, s); break;
            case 3: launch_conv_k<T, 3>(p, x, w, st_in, o0, o1, o2, s); break;
            case 4: launch_conv_k<T, 4>(p, x, w, st_in, o0, o1, o2, s); break;
            case 5: launch_conv_k<T, 5>(p, x, w, st_in, o0, o1, o2, s); break;
            case 6: launch_conv_k<T, 6>(p, x, w, st_in, o0, o1, o2, s); break;
            case 7: launch_conv_k<T, 7>(p, x, w, st_in, o0, o1, o2, s); break;
            case 8: launch_conv_k<T, 8>(p, x, w, st_in, o0, o1, o2, s); break;
            default: return cudaErrorInvalidValue;
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (st_out != nullptr && p.n_seqs > 0) {
        const int64_t n = static_cast<int64_t>(p.n_seqs) * p.channels;
        conv_state_kernel<T><<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
            p, static_cast<const T*>(x), st_in, st_out);
    }
    return cudaGetLastError();
}

}  // namespace

int conv_max_taps() { return kMaxTaps; }

cudaError_t launch_causal_conv1d(int dtype, int32_t n_seqs, int64_t tokens, int32_t seq_len,
                                 const int32_t* cu_seqlens, int32_t channels, int32_t taps,
                                 int32_t split0, int32_t split1, int32_t silu, const void* x,
                                 const void* weight, const float* state_in, void* out0,
                                 void* out1, void* out2, float* state_out, cudaStream_t s) {
    const Conv p{n_seqs, tokens, seq_len, cu_seqlens, channels, taps, split0, split1, silu};
    if (dtype == GDR_DTYPE_BF16)
        return launch_conv_t<__nv_bfloat16>(p, x, weight, state_in, out0, out1, out2, state_out,
                                            s);
    if (dtype == GDR_DTYPE_F16)
        return launch_conv_t<__half>(p, x, weight, state_in, out0, out1, out2, state_out, s);
    return launch_conv_t<float>(p, x, weight, state_in, out0, out1, out2, state_out, s);
}

cudaError_t launch_gates(int dtype, int64_t n, int heads, const void* a, const void* b,
                         const float* a_log, const float* dt_bias, float* g, float* beta,
                         cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (dtype == GDR_DTYPE_BF16)
        gates_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, s>>>(
            n, heads, static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
            a_log, dt_bias, g, beta);
    else if (dtype == GDR_DTYPE_F16)
        gates_kernel<__half><<<grid_for(n, 256), 256, 0, s>>>(
            n, heads, static_cast<const __half*>(a), static_cast<const __half*>(b), a_log,
            dt_bias, g, beta);
    else
        gates_kernel<float><<<grid_for(n, 256), 256, 0, s>>>(
            n, heads, static_cast<const float*>(a), static_cast<const float*>(b), a_log, dt_bias,
            g, beta);
    return cudaGetLastError();
}

cudaError_t launch_gated_norm(int dtype, int64_t rows, int width, const void* x, const void* z,
                              const float* weight, float eps, void* out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(z) |
                         reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(weight);
    if ((dtype == GDR_DTYPE_BF16 || dtype == GDR_DTYPE_F16) && width == 128 && (al & 15) == 0) {
        const int64_t warps = (rows + kNormRows - 1) / kNormRows;
        const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
        if (dtype == GDR_DTYPE_BF16)
            gated_norm_16b_128<__nv_bfloat16><<<grid, 256, 0, s>>>(
                rows, static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z),
                weight, eps, static_cast<__nv_bfloat16*>(out));
        else
            gated_norm_16b_128<__half><<<grid, 256, 0, s>>>(
                rows, static_cast<const __half*>(x), static_cast<const __half*>(z), weight, eps,
                static_cast<__half*>(out));
        return cudaGetLastError();
    }
    const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
    if (dtype == GDR_DTYPE_BF16)
        gated_norm_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
            rows, width, static_cast<const __nv_bfloat16*>(x),
            static_cast<const __nv_bfloat16*>(z), weight, eps, static_cast<__nv_bfloat16*>(out));
    else if (dtype == GDR_DTYPE_F16)
        gated_norm_kernel<__half><<<grid, 256, 0, s>>>(
            rows, width, static_cast<const __half*>(x), static_cast<const __half*>(z), weight, eps,
            static_cast<__half*>(out));
    else
        gated_norm_kernel<float><<<grid, 256, 0, s>>>(rows, width, static_cast<const float*>(x),
                                                      static_cast<const float*>(z), weight, eps,
                                                      static_cast<float*>(out));
    return cudaGetLastError();
}

cudaError_t launch_reorder(const void* src, void* dst, const int32_t* sources, int32_t rows,
                           int32_t src_rows, size_t row_bytes, cudaStream_t s) {
    if (rows == 0 || row_bytes == 0) return cudaSuccess;
    const uintptr_t al = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst);
    if (row_bytes % 16 == 0 && (al & 15) == 0) {
        const int64_t words = static_cast<int64_t>(row_bytes / 16);
        reorder_kernel<uint4><<<grid_for(rows * words, 256), 256, 0, s>>>(
            static_cast<const uint4*>(src), static_cast<uint4*>(dst), sources, rows, src_rows,
            words);
    } else {
        const int64_t words = static_cast<int64_t>(row_bytes / 4);
        reorder_kernel<uint32_t><<<grid_for(rows * words, 256), 256, 0, s>>>(
            static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), sources, rows,
            src_rows, words);
    }
    return cudaGetLastError();
}

}  // namespace gdr
