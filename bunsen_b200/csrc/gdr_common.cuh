// Shared device helpers and the launch descriptor every kernel receives.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdr.h"

namespace gdr {

// What a kernel needs to address one (sequence, head) of a call. Built on
// the host from gdr_params by the entry points in gdr_api.cu.
struct Problem {
    int32_t n_seqs;           // sequences (dense: B)
    int32_t seq_len;          // dense T (cu_seqlens == nullptr), else T_total
    const int32_t* cu_seqlens;  // nullptr: dense, sequence s = [s*T, (s+1)*T)
    int32_t heads_qk, heads_v, group;  // group = H_v / H_qk
    int32_t d_k, d_v, chunk;
    int32_t use_l2norm;
    float l2norm_eps;
    float q_scale;  // 1 / sqrt(d_k)
    // Steps of the layer fused into the rule (off while the pointers are
    // null): g and beta from the projections a, b [T, H_v] (gated_delta_net.rs:
    // 422-426), and the gated RMS norm of the output with z [T, H_v, d_v] in
    // the output's dtype and its weight [d_v] (:439-440).
    const void* gate_a = nullptr;
    const void* gate_b = nullptr;
    const float* a_log = nullptr;
    const float* dt_bias = nullptr;
    int32_t gate_dtype = GDR_DTYPE_F32;  // gdr_dtype of a and b
    int32_t gate_bf16 = 0;               // gate_dtype == GDR_DTYPE_BF16
    const void* norm_z = nullptr;
    const float* norm_w = nullptr;
    float norm_eps = 0.f;
};

// [start, end) of sequence s in the packed token axis. Offsets are clamped
// to [0, T_total] so a malformed cu_seqlens can never address outside the
// caller's buffers.
__device__ __forceinline__ void seq_span(const Problem& p, int s, int64_t& start, int64_t& end) {
    if (p.cu_seqlens == nullptr) {
        start = static_cast<int64_t>(s) * p.seq_len;
        end = start + p.seq_len;
        return;
    }
    int64_t a = p.cu_seqlens[s], b = p.cu_seqlens[s + 1];
    a = a < 0 ? 0 : (a > p.seq_len ? p.seq_len : a);
    b = b < a ? a : (b > p.seq_len ? p.seq_len : b);
    start = a;
    end = b;
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) {
    return __float2half_rn(x);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// 1 / (sqrt(sum x^2 + eps)), or 1 without the norm: bunsen's l2norm factor
// (delta_rule.rs:112-123), applied as a multiplication.
__device__ __forceinline__ float l2_factor(const Problem& p, float sumsq) {
    return p.use_l2norm ? 1.0f / sqrtf(sumsq + p.l2norm_eps) : 1.0f;
}

// The layer's gates from its projections (gated_delta_net.rs:422-426):
// g = -exp(A_log) softplus(a + dt_bias) in f32 (the layer widens a, A_log and
// dt_bias to f32 first); beta = sigmoid(b) on the projection's own tensor, so
// its value is rounded to the projection's dtype (bf16 in a bf16 model) before
// the rule widens it back to f32.
__device__ __forceinline__ float gate_g(float a, float a_log, float dt_bias) {
    const float x = a + dt_bias;
    const float sp = x > 20.f ? x : log1pf(expf(x));
    return -expf(a_log) * sp;
}
__device__ __forceinline__ float gate_beta(float b, int32_t dtype) {
    const float s = 1.f / (1.f + expf(-b));
    return dtype == GDR_DTYPE_BF16  ? __bfloat162float(__float2bfloat16_rn(s))
           : dtype == GDR_DTYPE_F16 ? __half2float(__float2half_rn(s))
                                    : s;
}

__device__ __forceinline__ float load_gate_input(const void* base, int64_t i, int32_t dtype) {
    return dtype == GDR_DTYPE_BF16  ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i])
           : dtype == GDR_DTYPE_F16 ? __half2float(static_cast<const __half*>(base)[i])
                                    : static_cast<const float*>(base)[i];
}

// g and beta of position-and-head index i = t * H_v + h: from the call's
// arrays, or produced from the projections when the layer's gates are fused.
__device__ __forceinline__ void rule_gates(const Problem& p, const float* g, const float* beta,
                                           int64_t i, int h, float& gi, float& bi) {
    if (p.gate_a != nullptr) {
        gi = gate_g(load_gate_input(p.gate_a, i, p.gate_dtype), p.a_log[h], p.dt_bias[h]);
        bi = gate_beta(load_gate_input(p.gate_b, i, p.gate_dtype), p.gate_dtype);
    } else {
        gi = g[i];
        bi = beta[i];
    }
}

// x sigmoid(x) = x / (1 + e^-x), written so neither side cancels: with
// u = e^-|x| (ex2.approx) and r = 1 / (1 + u) (rcp.approx), sigmoid(x) is r
// for x >= 0 and u r below. Relative error below 1e-6 for |x| < 10 and below
// 4e-6 for |x| < 100 (the rounding of the exponent's argument); the result
// underflows to -0 below x = -87.
__device__ __forceinline__ float silu(float x) {
    float u, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(u) : "f"(-1.44269504f * fabsf(x)));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + u));
    return x * (x >= 0.f ? r : u * r);
}

}  // namespace gdr
