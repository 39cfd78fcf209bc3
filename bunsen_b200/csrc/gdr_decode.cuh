// The d_k = d_v = 128 recurrent rule for one (sequence, value head), as a
// device function of a 256-thread CTA: the body of gdr_recurrent's fast
// kernel and of gdr_mixed's decode rows.
//
// GatedDeltaRule::recurrent (delta_rule.rs:182-209) per position t:
//   S <- exp(g_t) S;  read = k_t^T S;  delta = (v_t - read) beta_t;
//   S <- S + k_t delta^T;  o_t = q_t^T S
// Bandwidth bound: the f32 state is read from HBM once and written once (64
// KiB each way). Warp w holds state rows w, w+8, ..., w+120 and lane l
// columns 4l..4l+3 in registers, so every state access is a 128-bit load or
// store and a warp touches one whole 512-byte row per instruction. The two
// reductions over d_k (k^T S and q^T S) share one pass: o = q^T S_decayed +
// delta (q . k), which is q^T S after the rank-one update.
#pragma once

#include "gdr_common.cuh"

namespace gdr {

constexpr int kDecD = 128;
constexpr int kDecWarps = 8;
constexpr int kDecRowsPerWarp = kDecD / kDecWarps;  // 16 state rows per thread

struct DecodeSmem {
    float qk_raw[2][kDecD];            // this position's q and k
    float red[2][kDecWarps][kDecD];    // per-warp partial k^T S, q^T S
    float delta_s[kDecD];
    float scal[4];                     // |q|^2, |k|^2, -, q.k
    float nrm[4];                      // per-warp sums of squares of the output
};

using DecodeState = float[kDecRowsPerWarp][4];

// This thread's part of a [128, 128] f32 state (global or shared memory,
// row-major): rows warp + 8 r, columns 4 lane .. 4 lane + 3.
__device__ __forceinline__ void decode_load_state(const float* src, DecodeState& st) {
    const int warp = threadIdx.x >> 5, col = 4 * (threadIdx.x & 31);
#pragma unroll
    for (int r = 0; r < kDecRowsPerWarp; ++r) {
        const float4 x = *reinterpret_cast<const float4*>(src + (warp + kDecWarps * r) * kDecD + col);
        st[r][0] = x.x; st[r][1] = x.y; st[r][2] = x.z; st[r][3] = x.w;
    }
}

__device__ __forceinline__ void decode_store_state(float* dst, const DecodeState& st) {
    const int warp = threadIdx.x >> 5, col = 4 * (threadIdx.x & 31);
#pragma unroll
    for (int r = 0; r < kDecRowsPerWarp; ++r)
        *reinterpret_cast<float4*>(dst + (warp + kDecWarps * r) * kDecD + col) =
            make_float4(st[r][0], st[r][1], st[r][2], st[r][3]);
}

// This thread's inputs of position t of value head h, as loaded (converted
// where they are used, so that a load issued a position ahead is not waited
// for at once): one element of q (threads 0-127) or k (128-255), and, for
// threads 0-127, one of v and of the gated norm's z; g and beta, or, with the
// layer's gates fused, the bits of the projections a and b.
template <typename T>
struct DecodeIn {
    T qk, v, z;
    uint32_t ga, gb;
};

__device__ __forceinline__ uint32_t gate_bits(const void* base, int64_t i, int32_t dtype) {
    uint32_t x;
    if (dtype == GDR_DTYPE_F32)
        x = __float_as_uint(static_cast<const float*>(base)[i]);
    else
        x = static_cast<const uint16_t*>(base)[i];
    return x;
}

__device__ __forceinline__ float gate_value(uint32_t x, int32_t dtype) {
    return dtype == GDR_DTYPE_F32    ? __uint_as_float(x)
           : dtype == GDR_DTYPE_BF16 ? __uint_as_float(x << 16)
                                     : __half2float(__ushort_as_half(static_cast<unsigned short>(x)));
}

template <typename T>
__device__ __forceinline__ DecodeIn<T> decode_in(const Problem& p, const T* __restrict__ q,
                                                 const T* __restrict__ k,
                                                 const T* __restrict__ v,
                                                 const float* __restrict__ g,
                                                 const float* __restrict__ beta, int64_t t,
                                                 int h) {
    const int tid = threadIdx.x;
    DecodeIn<T> in;
    const int64_t qk_off = (t * p.heads_qk + h / p.group) * kDecD;
    in.qk = ((tid < 128) ? q : k)[qk_off + (tid & 127)];
    const int64_t orow = (t * p.heads_v + h) * kDecD;
    in.v = v[orow + (tid & 127)];
    in.z = from_f32<T>(0.f);
    if (p.norm_z != nullptr) in.z = static_cast<const T*>(p.norm_z)[orow + (tid & 127)];
    const int64_t i = t * p.heads_v + h;
    if (p.gate_a != nullptr) {
        in.ga = gate_bits(p.gate_a, i, p.gate_dtype);
        in.gb = gate_bits(p.gate_b, i, p.gate_dtype);
    } else {
        in.ga = __float_as_uint(g[i]);
        in.gb = __float_as_uint(beta[i]);
    }
    return in;
}

// g and beta of a position from its loaded inputs (rule_gates' arithmetic).
template <typename T>
__device__ __forceinline__ void decode_gates(const Problem& p, const DecodeIn<T>& in, int h,
                                             float& gt, float& bt) {
    if (p.gate_a != nullptr) {
        gt = gate_g(gate_value(in.ga, p.gate_dtype), p.a_log[h], p.dt_bias[h]);
        bt = gate_beta(gate_value(in.gb, p.gate_dtype), p.gate_dtype);
    } else {
        gt = __uint_as_float(in.ga);
        bt = __uint_as_float(in.gb);
    }
}

// The rule over positions [t0, t1) of value head h, the state in registers.
// `in0` holds position t0's inputs (decode_in); each position's loads for the
// next one are issued before its own arithmetic, so no position waits for a
// global round trip of its own. `smem` holds a DecodeSmem.
template <typename T>
__device__ __forceinline__ void decode_positions(const Problem& p, const T* __restrict__ q,
                                                 const T* __restrict__ k,
                                                 const T* __restrict__ v,
                                                 const float* __restrict__ g,
                                                 const float* __restrict__ beta, int64_t t0,
                                                 int64_t t1, int h, DecodeState& st,
                                                 T* __restrict__ out, uint8_t* smem,
                                                 DecodeIn<T> in0) {
    constexpr int kD = kDecD, kWarps = kDecWarps, kRowsPerWarp = kDecRowsPerWarp;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto& sh = *reinterpret_cast<DecodeSmem*>(smem);
    auto& qk_raw = sh.qk_raw;
    auto& red = sh.red;
    auto& delta_s = sh.delta_s;
    auto& scal = sh.scal;
    const int col = 4 * lane;
    DecodeIn<T> in = in0;
    for (int64_t t = t0; t < t1; ++t) {
        // q and k of this position, raw, into shared memory; the next
        // position's inputs on their way.
        qk_raw[tid >> 7][tid & 127] = to_f32(in.qk);
        const bool more = t + 1 < t1;
        DecodeIn<T> nxt;
        if (more) nxt = decode_in(p, q, k, v, g, beta, t + 1, h);
        float gt, bt;
        decode_gates(p, in, h, gt, bt);
        const float decay = __expf(gt);
        __syncthreads();
        if (warp < 3) {  // |q|^2, |k|^2, q.k
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = qk_raw[warp == 1 ? 1 : 0][col + i];
                b[i] = qk_raw[warp == 0 ? 0 : 1][col + i];
            }
            float acc = a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3];
            acc = warp_sum(acc);
            if (lane == 0) scal[warp == 2 ? 3 : warp] = acc;  // 0: |q|^2 1: |k|^2 3: q.k
        }
        __syncthreads();
        const float fq = l2_factor(p, scal[0]) * p.q_scale;
        const float fk = l2_factor(p, scal[1]);
        float pk[4] = {0.f, 0.f, 0.f, 0.f}, pq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            const int row = warp + kWarps * r;
            const float kr = qk_raw[1][row] * fk, qr = qk_raw[0][row] * fq;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                st[r][c] *= decay;
                pk[c] = fmaf(kr, st[r][c], pk[c]);
                pq[c] = fmaf(qr, st[r][c], pq[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            red[0][warp][col + c] = pk[c];
            red[1][warp][col + c] = pq[c];
        }
        __syncthreads();
        float o = 0.f;
        const int64_t orow = (t * p.heads_v + h) * kD;
        if (tid < kD) {
            float read = 0.f, qs = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                read += red[0][w][tid];
                qs += red[1][w][tid];
            }
            const float d = (to_f32(in.v) - read) * bt;
            delta_s[tid] = d;
            const float qk_dot = scal[3] * fq * fk;
            o = fmaf(d, qk_dot, qs);
            if (p.norm_z == nullptr) {
                out[orow + tid] = from_f32<T>(o);
            } else {  // the norm reads the output in its own dtype
                o = to_f32(from_f32<T>(o));
                const float ss = warp_sum(o * o);
                if (lane == 0) sh.nrm[warp] = ss;
            }
        }
        __syncthreads();
        if (p.norm_z != nullptr && tid < kD) {  // gated RMS norm of the 128 outputs
            const float r = rsqrtf((sh.nrm[0] + sh.nrm[1] + sh.nrm[2] + sh.nrm[3]) / kD + p.norm_eps);
            out[orow + tid] = from_f32<T>(o * r * p.norm_w[tid] * silu(to_f32(in.z)));
        }
        float dl[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) dl[c] = delta_s[col + c];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            const float kr = qk_raw[1][warp + kWarps * r] * fk;
#pragma unroll
            for (int c = 0; c < 4; ++c) st[r][c] = fmaf(kr, dl[c], st[r][c]);
        }
        __syncthreads();  // qk_raw, red and delta_s are rewritten next position
        if (more) in = nxt;
    }

}

// Positions [t0, t1) of value head h; state_in may be null (zeros) and may
// equal state_out. `smem` holds a DecodeSmem.
template <typename T>
__device__ __forceinline__ void recurrent_d128_item(const Problem& p, const T* __restrict__ q,
                                                    const T* __restrict__ k,
                                                    const T* __restrict__ v,
                                                    const float* __restrict__ g,
                                                    const float* __restrict__ beta,
                                                    int64_t t0, int64_t t1, int h,
                                                    const float* state_in, T* __restrict__ out,
                                                    float* state_out, uint8_t* smem) {
    DecodeState st;
    if (state_in != nullptr) {
        decode_load_state(state_in, st);
    } else {
#pragma unroll
        for (int r = 0; r < kDecRowsPerWarp; ++r) st[r][0] = st[r][1] = st[r][2] = st[r][3] = 0.f;
    }
    DecodeIn<T> in0{};
    if (t0 < t1) in0 = decode_in(p, q, k, v, g, beta, t0, h);
    decode_positions<T>(p, q, k, v, g, beta, t0, t1, h, st, out, smem, in0);
    decode_store_state(state_out, st);
}

}  // namespace gdr
