// GatedDeltaRule::chunked (delta_rule.rs:223-310) in f32 on CUDA cores for the
// production head size: d_k = d_v = 128, chunk 64, q/k/v in f32, f16 or bf16.
//
// Every product is an f32 FMA, as in bunsen's f32 rule (and in its f16 runs,
// which it widens to f32, burner/tensor/widening.rs:58-60). One CTA of 256
// threads per (sequence, value head) walks the sequence's chunks with the
// [128, 128] state in shared memory. Each product of a chunk is register-
// tiled: a thread owns a 4 x 8 (or 8 x 8) block of the result, consecutive
// rows and columns in two groups of four. The left operands that a k step
// reads down a column (the inverse X and the intra matrix) are kept
// transposed, so each k step loads one or two 16-byte vectors of them (a few
// scalars where the operand is row-major) and two 16-byte vectors of the right
// operand for 32 or 64 FMAs; a warp's vector loads cover consecutive 16-byte
// pieces of one row (no bank conflicts).
//
// Per chunk of C = 64 positions (zero-padded past the sequence end, where
// g = beta = 0 and nothing is written, delta_rule.rs:241-262):
//   1. q, k rows L2-normalised (q also / sqrt(d_k)), v scaled by beta,
//      gamma = cumsum(g)                                    (:151-154, :263-272)
//   2. Gram K K^T and Q K^T; a = -strict_lower(beta K K^T o Gamma),
//      intra = lower(Q K^T o Gamma)                          (:273-279)
//   3. X = (I + L)^-1 by forward substitution, one column per thread of the
//      first two warps                                       (:337-351)
//   4. U = X (beta V), W = X diag(beta e^gamma) K            (:283-285)
//   5. (Q S) diag(e^gamma) and W S, one pass over S
//   6. V_new = U - W S                                       (:299-300)
//   7. O = Q_c S + intra V_new; S <- e^gamma_C S + (K e^(gamma_C - gamma))^T V_new
#include "gdr_common.cuh"

namespace gdr {

namespace {

constexpr int kC = 64, kD = 128, kThreads = 256;
constexpr int kLd = kD + 4;   // row stride (floats) of the [.][128] arrays
constexpr int kLc = kC + 4;   // row stride of the [64][64] arrays

struct F32Smem {
    float S[kD * kLd];   // the state, [d_k][d_v]
    float Q[kC * kLd];   // normalised, scaled q; then V_new
    float K[kC * kLd];   // normalised k
    float V[kC * kLd];   // beta v; then W
    float A[kC * kLc];   // -L, then X = (I + L)^-1
    float I[kC * kLc];   // intra
    float gam[kC];  // cumulative log decay within the chunk
    float bet[kC];  // beta
    float eg[kC];   // e^gamma
    float wf[kC];   // beta e^gamma
    float rr[kC];   // e^(gamma_C - gamma)
};

// Global -> f32 helpers for 4 consecutive elements.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__half* p, float4 v) {
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

// acc[a][8] += x[a] * (row[n0 .. n0+3], row[n0+64 .. n0+67]) for the four rows a.
__device__ __forceinline__ void fma_4x8(float (&acc)[4][8], const float (&x)[4], const float* row,
                                        int n0) {
    const float4 b0 = *reinterpret_cast<const float4*>(row + n0);
    const float4 b1 = *reinterpret_cast<const float4*>(row + n0 + 64);
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[a][c] = fmaf(x[a], bv[c], acc[a][c]);
}

// The same for eight rows.
__device__ __forceinline__ void fma_8x8(float (&acc)[8][8], const float (&x)[8], const float* row,
                                        int n0) {
    const float4 b0 = *reinterpret_cast<const float4*>(row + n0);
    const float4 b1 = *reinterpret_cast<const float4*>(row + n0 + 64);
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[a][c] = fmaf(x[a], bv[c], acc[a][c]);
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    return fmaf(a.w, b.w, acc);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
chunked_f32_d128(Problem p, const T* __restrict__ q, const T* __restrict__ k,
                 const T* __restrict__ v, const float* __restrict__ g,
                 const float* __restrict__ beta, const float* state_in, T* __restrict__ out,
                 float* state_out) {
    extern __shared__ __align__(16) uint8_t f32_smem_raw[];
    F32Smem& sm = *reinterpret_cast<F32Smem*>(f32_smem_raw);
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int ti = tid >> 4, tj = tid & 15;  // rows 4 ti + a, columns n0 .. and n0 + 64 ..
    const int n0 = 4 * tj;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t len = t1 - t0;
    const int64_t hs = (static_cast<int64_t>(s) * p.heads_v + h) * kD * kD;
    const int hq = h / p.group;
    for (int e = tid; e < kD * kD / 4; e += kThreads) {
        const int x = e >> 5, c4 = (e & 31) * 4;
        store4(sm.S + x * kLd + c4,
               state_in ? load4(state_in + hs + x * kD + c4) : make_float4(0.f, 0.f, 0.f, 0.f));
    }
    const int n_chunks = static_cast<int>((len + kC - 1) / kC);
#pragma unroll 1
    for (int ci = 0; ci < n_chunks; ++ci) {
        const int64_t base = t0 + static_cast<int64_t>(ci) * kC;
        const int64_t left = len - static_cast<int64_t>(ci) * kC;
        const int valid = static_cast<int>(left < kC ? left : kC);
        // 1. Rows of q, k, v (zeros past the end), g and beta, gamma.
        for (int e = tid; e < kC * kD / 4; e += kThreads) {
            const int r = e >> 5, c4 = (e & 31) * 4;
            float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv, vv = qv;
            if (r < valid) {
                const int64_t qk = ((base + r) * p.heads_qk + hq) * kD + c4;
                qv = load4(q + qk);
                kv = load4(k + qk);
                vv = load4(v + ((base + r) * p.heads_v + h) * kD + c4);
            }
            store4(sm.Q + r * kLd + c4, qv);
            store4(sm.K + r * kLd + c4, kv);
            store4(sm.V + r * kLd + c4, vv);
        }
        if (warp == 0) {
            const int r0 = 2 * lane, r1 = r0 + 1;
            const float g0 = r0 < valid ? g[(base + r0) * p.heads_v + h] : 0.f;
            const float g1 = r1 < valid ? g[(base + r1) * p.heads_v + h] : 0.f;
            sm.bet[r0] = r0 < valid ? beta[(base + r0) * p.heads_v + h] : 0.f;
            sm.bet[r1] = r1 < valid ? beta[(base + r1) * p.heads_v + h] : 0.f;
            float incl = g0 + g1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            sm.gam[r0] = incl - g1;
            sm.gam[r1] = incl;
        }
        __syncthreads();
        // prepare (delta_rule.rs:151-154): rows of q and k normalised, q scaled;
        // one warp per row, four features per lane. v scaled by beta.
        for (int r = warp; r < 2 * kC; r += kThreads / 32) {
            float* row = (r < kC ? sm.Q + r * kLd : sm.K + (r - kC) * kLd) + 4 * lane;
            float4 xv = *reinterpret_cast<float4*>(row);
            const float ss = warp_sum(dot4(xv, xv, 0.f));
            const float f = l2_factor(p, ss) * (r < kC ? p.q_scale : 1.f);
            xv.x *= f;
            xv.y *= f;
            xv.z *= f;
            xv.w *= f;
            *reinterpret_cast<float4*>(row) = xv;
        }
        for (int e = tid; e < kC * kD / 4; e += kThreads) {
            const int r = e >> 5, c4 = (e & 31) * 4;
            float4* pv = reinterpret_cast<float4*>(sm.V + r * kLd + c4);
            const float b = sm.bet[r];
            float4 xv = *pv;
            xv.x *= b;
            xv.y *= b;
            xv.z *= b;
            xv.w *= b;
            *pv = xv;
        }
        if (tid < kC) {
            const float gt = sm.gam[tid];
            const float eg = __expf(gt);
            sm.eg[tid] = eg;
            sm.wf[tid] = sm.bet[tid] * eg;
            sm.rr[tid] = __expf(sm.gam[kC - 1] - gt);
        }
        __syncthreads();
        // 2. Gram products and the masked, decayed L and intra.
        {
            float kk[4][4] = {}, qk[4][4] = {};
#pragma unroll 2
            for (int x = 0; x < kD; x += 4) {
                float4 ki[4], qi[4], kj[4];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    ki[a] = *reinterpret_cast<const float4*>(sm.K + (ti + 16 * a) * kLd + x);
                    qi[a] = *reinterpret_cast<const float4*>(sm.Q + (ti + 16 * a) * kLd + x);
                    kj[a] = *reinterpret_cast<const float4*>(sm.K + (tj + 16 * a) * kLd + x);
                }
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        kk[a][b] = dot4(ki[a], kj[b], kk[a][b]);
                        qk[a][b] = dot4(qi[a], kj[b], qk[a][b]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int i = ti + 16 * a, j = tj + 16 * b;
                    const float dec = j <= i ? __expf(sm.gam[i] - sm.gam[j]) : 0.f;
                    sm.A[i * kLc + j] = j < i ? -(sm.bet[i] * kk[a][b]) * dec : 0.f;
                    sm.I[j * kLc + i] = qk[a][b] * dec;  // transposed: I^T
                }
        }
        __syncthreads();
        // 3. X = (I + L)^-1, column m by thread m: X[r][m] = delta_rm +
        //    sum_{s < r} a[r][s] X[s][m], a = -L (rows of a read in order).
        {
            float xc[kC];
            if (tid < kC) {
#pragma unroll
                for (int r = 0; r < kC; ++r) xc[r] = r == tid ? 1.f : 0.f;
#pragma unroll
                for (int s2 = 0; s2 < kC - 1; ++s2)
#pragma unroll
                    for (int r = s2 + 1; r < kC; ++r) xc[r] = fmaf(sm.A[r * kLc + s2], xc[s2], xc[r]);
            }
            __syncthreads();
            if (tid < kC) {  // X^T: column tid of X is row tid here
#pragma unroll
                for (int r = 0; r < kC; r += 4)
                    store4(sm.A + tid * kLc + r, make_float4(xc[r], xc[r + 1], xc[r + 2], xc[r + 3]));
            }
        }
        __syncthreads();
        // 4. U = X (beta V) and W = X diag(beta e^gamma) K, this thread's rows
        //    4 ti .. 4 ti + 3 and columns n0 .. n0 + 3, n0 + 64 .. n0 + 67.
        float u[4][8] = {}, w[4][8] = {};
#pragma unroll 4
        for (int j = 0; j < kC; ++j) {
            const float wj = sm.wf[j];
            const float4 x4 = *reinterpret_cast<const float4*>(sm.A + j * kLc + 4 * ti);
            const float xa[4] = {x4.x, x4.y, x4.z, x4.w};
            float xw[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xw[a] = xa[a] * wj;
            fma_4x8(u, xa, sm.V + j * kLd, n0);
            fma_4x8(w, xw, sm.K + j * kLd, n0);
        }
        __syncthreads();  // beta V is read: W goes into its buffer
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float* row = sm.V + (4 * ti + a) * kLd;
            store4(row + n0, make_float4(w[a][0], w[a][1], w[a][2], w[a][3]));
            store4(row + n0 + 64, make_float4(w[a][4], w[a][5], w[a][6], w[a][7]));
        }
        __syncthreads();
        // 5. (Q S) and (W S) in one pass over the state's rows; 6. V_new = U - W S.
        float o[4][8] = {};
        {
            float ws[4][8] = {};
#pragma unroll 2
            for (int x = 0; x < kD; ++x) {
                float qa[4], wa[4];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    qa[a] = sm.Q[(4 * ti + a) * kLd + x];
                    wa[a] = sm.V[(4 * ti + a) * kLd + x];
                }
                fma_4x8(o, qa, sm.S + x * kLd, n0);
                fma_4x8(ws, wa, sm.S + x * kLd, n0);
            }
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float eg = sm.eg[4 * ti + a];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    u[a][c] -= ws[a][c];
                    o[a][c] *= eg;
                }
            }
        }
        __syncthreads();  // Q and W are read: V_new goes into Q's buffer
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float* row = sm.Q + (4 * ti + a) * kLd;
            store4(row + n0, make_float4(u[a][0], u[a][1], u[a][2], u[a][3]));
            store4(row + n0 + 64, make_float4(u[a][4], u[a][5], u[a][6], u[a][7]));
        }
        __syncthreads();
        // 7. O = (e^gamma Q) S + intra V_new (rows past the end dropped) ...
#pragma unroll 4
        for (int j = 0; j < kC; ++j) {
            const float4 i4 = *reinterpret_cast<const float4*>(sm.I + j * kLc + 4 * ti);
            const float ia[4] = {i4.x, i4.y, i4.z, i4.w};
            fma_4x8(o, ia, sm.Q + j * kLd, n0);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int i = 4 * ti + a;
            if (i < valid) {
                T* dst = out + ((base + i) * p.heads_v + h) * kD;
                store4(dst + n0, make_float4(o[a][0], o[a][1], o[a][2], o[a][3]));
                store4(dst + n0 + 64, make_float4(o[a][4], o[a][5], o[a][6], o[a][7]));
            }
        }
        // ... and S <- e^gamma_C S + (K e^(gamma_C - gamma))^T V_new, rows 8 ti .. 8 ti + 7.
        {
            const float decay = __expf(sm.gam[kC - 1]);
            float st[8][8];
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                const float* row = sm.S + (8 * ti + a) * kLd;
                const float4 b0 = *reinterpret_cast<const float4*>(row + n0);
                const float4 b1 = *reinterpret_cast<const float4*>(row + n0 + 64);
                st[a][0] = b0.x * decay; st[a][1] = b0.y * decay;
                st[a][2] = b0.z * decay; st[a][3] = b0.w * decay;
                st[a][4] = b1.x * decay; st[a][5] = b1.y * decay;
                st[a][6] = b1.z * decay; st[a][7] = b1.w * decay;
            }
#pragma unroll 2
            for (int r = 0; r < kC; ++r) {
                const float f = sm.rr[r];
                const float4 k0 = *reinterpret_cast<const float4*>(sm.K + r * kLd + 8 * ti);
                const float4 k1 = *reinterpret_cast<const float4*>(sm.K + r * kLd + 8 * ti + 4);
                const float ka[8] = {k0.x * f, k0.y * f, k0.z * f, k0.w * f,
                                     k1.x * f, k1.y * f, k1.z * f, k1.w * f};
                fma_8x8(st, ka, sm.Q + r * kLd, n0);
            }
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                float* row = sm.S + (8 * ti + a) * kLd;
                store4(row + n0, make_float4(st[a][0], st[a][1], st[a][2], st[a][3]));
                store4(row + n0 + 64, make_float4(st[a][4], st[a][5], st[a][6], st[a][7]));
            }
        }
        __syncthreads();
    }
    for (int e = tid; e < kD * kD / 4; e += kThreads) {
        const int x = e >> 5, c4 = (e & 31) * 4;
        store4(state_out + hs + x * kD + c4, load4(sm.S + x * kLd + c4));
    }
}

}  // namespace

bool chunked_f32_d128_supports(const Problem& p, int dtype, const void* q, const void* k,
                               const void* v, const void* out, const float* state_in,
                               const float* state_out) {
    const uintptr_t need = dtype == GDR_DTYPE_F32 ? 15 : 7;
    const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
    const uintptr_t als = reinterpret_cast<uintptr_t>(state_in) |
                          reinterpret_cast<uintptr_t>(state_out);
    return p.d_k == kD && p.d_v == kD && p.chunk == kC && (al & need) == 0 && (als & 15) == 0;
}

template <typename T>
static cudaError_t launch_f32_t(const Problem& p, const void* q, const void* k, const void* v,
                                const float* g, const float* beta, const float* state_in,
                                void* out, float* state_out, cudaStream_t stream) {
    const int smem = static_cast<int>(sizeof(F32Smem));
    cudaError_t e = cudaFuncSetAttribute(chunked_f32_d128<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    chunked_f32_d128<T><<<dim3(p.heads_v, p.n_seqs), kThreads, smem, stream>>>(
        p, static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g, beta,
        state_in, static_cast<T*>(out), state_out);
    return cudaGetLastError();
}

cudaError_t launch_chunked_f32_d128(const Problem& p, int dtype, const void* q, const void* k,
                                    const void* v, const float* g, const float* beta,
                                    const float* state_in, void* out, float* state_out,
                                    cudaStream_t stream) {
    if (dtype == GDR_DTYPE_BF16)
        return launch_f32_t<__nv_bfloat16>(p, q, k, v, g, beta, state_in, out, state_out, stream);
    if (dtype == GDR_DTYPE_F16)
        return launch_f32_t<__half>(p, q, k, v, g, beta, state_in, out, state_out, stream);
    return launch_f32_t<float>(p, q, k, v, g, beta, state_in, out, state_out, stream);
}

}  // namespace gdr
