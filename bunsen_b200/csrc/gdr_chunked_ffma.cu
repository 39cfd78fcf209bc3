// GatedDeltaRule::chunked (delta_rule.rs:223-310) in f32 on CUDA cores.
//
// The f32 path: every product is an f32 FMA, so f32 runs agree with bunsen's
// f32 rule to f32 rounding. Any d_k, d_v <= 128 and chunk <= 64. One CTA of
// 256 threads per (sequence, value head) walks the sequence's chunks in
// order with the [d_k, d_v] state resident in shared memory.
//
// Per chunk of C positions (padded with zeros past the sequence end, which
// neither write nor decay, delta_rule.rs:241-262):
//   gamma = cumsum(g);  Gamma_ij = exp(gamma_i - gamma_j) for j <= i
//   L = strict_lower((beta k) k^T o Gamma);   intra = (q k^T) o Gamma
//   A = (I + L)^-1   (row forward substitution, delta_rule.rs:337-351)
//   U = A (beta v);  W = A (beta exp(gamma) k)
//   V_new = U - W S
//   O = (exp(gamma) q) S + intra V_new
//   S = exp(gamma_C) S + (exp(gamma_C - gamma) k)^T V_new
#include "gdr_common.cuh"

namespace gdr {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxC = 64;
constexpr int kMaxD = 128;
constexpr int kOwn = kMaxC * kMaxD / kThreads;  // [C, d] entries a thread owns

struct FfmaSmem {
    float* S;      // [dk][dv] the state
    float* Q;      // [C][dk]  normalised, scaled queries; later W
    float* K;      // [C][dk]  normalised keys
    float* V;      // [C][dv]  values; later U, then V_new
    float* A;      // [C][C]   -L, then (I + L)^-1
    float* I;      // [C][C]   intra
    float* gam;    // [C]      cumulative log decay
    float* bet;    // [C]      beta
    float* nxt;    // [C]      a row of the forward substitution
};

__host__ __device__ inline size_t ffma_smem_floats(int dk, int dv, int c) {
    return static_cast<size_t>(dk) * dv + 2 * c * dk + c * dv + 2 * c * c + 3 * c;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
chunked_ffma(Problem p, const T* __restrict__ q, const T* __restrict__ k,
             const T* __restrict__ v, const float* __restrict__ g,
             const float* __restrict__ beta, const float* state_in, T* __restrict__ out,
             float* state_out) {
    extern __shared__ float smem[];
    const int dk = p.d_k, dv = p.d_v, C = p.chunk;
    FfmaSmem sm;
    sm.S = smem;
    sm.Q = sm.S + dk * dv;
    sm.K = sm.Q + C * dk;
    sm.V = sm.K + C * dk;
    sm.A = sm.V + C * dv;
    sm.I = sm.A + C * C;
    sm.gam = sm.I + C * C;
    sm.bet = sm.gam + C;
    sm.nxt = sm.bet + C;

    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t len = t1 - t0;
    const int64_t head_state = (static_cast<int64_t>(s) * p.heads_v + h) * dk * dv;
    for (int e = tid; e < dk * dv; e += kThreads)
        sm.S[e] = state_in ? state_in[head_state + e] : 0.f;
    const int hq = h / p.group;
    const int n_chunks = static_cast<int>((len + C - 1) / C);

    for (int ci = 0; ci < n_chunks; ++ci) {
        const int64_t base = t0 + static_cast<int64_t>(ci) * C;
        // 1. The chunk, zero-padded past the sequence end.
        for (int e = tid; e < C * dk; e += kThreads) {
            const int r = e / dk, i = e % dk;
            const bool in = ci * static_cast<int64_t>(C) + r < len;
            const int64_t off = ((base + r) * p.heads_qk + hq) * dk + i;
            sm.Q[e] = in ? to_f32(q[off]) : 0.f;
            sm.K[e] = in ? to_f32(k[off]) : 0.f;
        }
        for (int e = tid; e < C * dv; e += kThreads) {
            const int r = e / dv, j = e % dv;
            const bool in = ci * static_cast<int64_t>(C) + r < len;
            sm.V[e] = in ? to_f32(v[((base + r) * p.heads_v + h) * dv + j]) : 0.f;
        }
        for (int r = tid; r < C; r += kThreads) {
            const bool in = ci * static_cast<int64_t>(C) + r < len;
            sm.gam[r] = in ? g[(base + r) * p.heads_v + h] : 0.f;
            sm.bet[r] = in ? beta[(base + r) * p.heads_v + h] : 0.f;
        }
        __syncthreads();
        // 2. prepare (delta_rule.rs:151-154): rows of q and k normalised, q
        //    scaled; one warp per row. Then the cumulative decay.
        for (int r = warp; r < 2 * C; r += kThreads / 32) {
            float* row = r < C ? sm.Q + r * dk : sm.K + (r - C) * dk;
            float acc = 0.f;
            for (int i = lane; i < dk; i += 32) acc = fmaf(row[i], row[i], acc);
            acc = warp_sum(acc);
            const float f = l2_factor(p, acc) * (r < C ? p.q_scale : 1.f);
            for (int i = lane; i < dk; i += 32) row[i] *= f;
        }
        if (tid == 0)
            for (int r = 1; r < C; ++r) sm.gam[r] += sm.gam[r - 1];
        __syncthreads();
        // 3. A = -strict_lower((beta k) k^T o Gamma), intra = (q k^T) o Gamma.
        for (int e = tid; e < C * C; e += kThreads) {
            const int i = e / C, j = e % C;
            float a = 0.f, in = 0.f;
            if (j <= i) {
                float kk = 0.f, qk = 0.f;
                for (int x = 0; x < dk; ++x) {
                    const float kj = sm.K[j * dk + x];
                    kk = fmaf(sm.K[i * dk + x], kj, kk);
                    qk = fmaf(sm.Q[i * dk + x], kj, qk);
                }
                const float decay = __expf(sm.gam[i] - sm.gam[j]);
                if (j < i) a = -(sm.bet[i] * kk) * decay;
                in = qk * decay;
            }
            sm.A[e] = a;
            sm.I[e] = in;
        }
        __syncthreads();
        // 4. Forward substitution, one row at a time (delta_rule.rs:344-349):
        //    a[i, :i] += sum_j a[i, j] a[j, :i].
        for (int i = 1; i < C; ++i) {
            if (tid < i) {
                float acc = 0.f;
                for (int j = 0; j < i; ++j) acc = fmaf(sm.A[i * C + j], sm.A[j * C + tid], acc);
                sm.nxt[tid] = sm.A[i * C + tid] + acc;
            }
            __syncthreads();
            if (tid < i) sm.A[i * C + tid] = sm.nxt[tid];
            __syncthreads();
        }
        for (int i = tid; i < C; i += kThreads) sm.A[i * C + i] = 1.f;
        __syncthreads();
        // 5. U = A (beta v) and the state part of the output,
        //    (exp(gamma) q) S, both into registers.
        float u[kOwn], o[kOwn];
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            u[m] = o[m] = 0.f;
            if (e < C * dv) {
                const int r = e / dv, c = e % dv;
                float acc = 0.f;
                for (int j = 0; j <= r; ++j)
                    acc = fmaf(sm.A[r * C + j], sm.V[j * dv + c] * sm.bet[j], acc);
                u[m] = acc;
                float os = 0.f;
                for (int x = 0; x < dk; ++x) os = fmaf(sm.Q[r * dk + x], sm.S[x * dv + c], os);
                o[m] = os * __expf(sm.gam[r]);
            }
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dv) sm.V[e] = u[m];
        }
        // 6. W = A (beta exp(gamma) k), into the queries' buffer.
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dk) {
                const int r = e / dk, x = e % dk;
                float acc = 0.f;
                for (int j = 0; j <= r; ++j)
                    acc = fmaf(sm.A[r * C + j],
                               sm.K[j * dk + x] * (sm.bet[j] * __expf(sm.gam[j])), acc);
                u[m] = acc;
            }
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dk) sm.Q[e] = u[m];
        }
        __syncthreads();
        // 7. V_new = U - W S.
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dv) {
                const int r = e / dv, c = e % dv;
                float ws = 0.f;
                for (int x = 0; x < dk; ++x) ws = fmaf(sm.Q[r * dk + x], sm.S[x * dv + c], ws);
                u[m] = sm.V[e] - ws;
            }
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dv) sm.V[e] = u[m];
        }
        __syncthreads();
        // 8. O = (exp(gamma) q) S + intra V_new, rows past the end dropped.
#pragma unroll
        for (int m = 0; m < kOwn; ++m) {
            const int e = tid + kThreads * m;
            if (e < C * dv) {
                const int r = e / dv, c = e % dv;
                float acc = o[m];
                for (int j = 0; j <= r; ++j) acc = fmaf(sm.I[r * C + j], sm.V[j * dv + c], acc);
                if (ci * static_cast<int64_t>(C) + r < len)
                    out[((base + r) * p.heads_v + h) * dv + c] = from_f32<T>(acc);
            }
        }
        // 9. S = exp(gamma_C) S + (exp(gamma_C - gamma) k)^T V_new.
        const float last = sm.gam[C - 1];
        const float chunk_decay = __expf(last);
        for (int e = tid; e < dk * dv; e += kThreads) {
            const int x = e / dv, c = e % dv;
            float acc = 0.f;
            for (int r = 0; r < C; ++r)
                acc = fmaf(sm.K[r * dk + x] * __expf(last - sm.gam[r]), sm.V[r * dv + c], acc);
            sm.S[e] = fmaf(sm.S[e], chunk_decay, acc);
        }
        __syncthreads();
    }
    for (int e = tid; e < dk * dv; e += kThreads) state_out[head_state + e] = sm.S[e];
}

}  // namespace

size_t chunked_ffma_smem_bytes(int dk, int dv, int c) {
    return sizeof(float) * ffma_smem_floats(dk, dv, c);
}

bool chunked_ffma_supports(int dk, int dv, int c) {
    return dk >= 1 && dv >= 1 && dk <= kMaxD && dv <= kMaxD && c >= 1 && c <= kMaxC &&
           chunked_ffma_smem_bytes(dk, dv, c) <= 227 * 1024;
}

template <typename T>
static cudaError_t launch_ffma_t(const Problem& p, const void* q, const void* k, const void* v,
                                 const float* g, const float* beta, const float* state_in,
                                 void* out, float* state_out, cudaStream_t stream) {
    const size_t smem = chunked_ffma_smem_bytes(p.d_k, p.d_v, p.chunk);
    cudaError_t e = cudaFuncSetAttribute(chunked_ffma<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    chunked_ffma<T><<<dim3(p.heads_v, p.n_seqs), kThreads, smem, stream>>>(
        p, static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g, beta,
        state_in, static_cast<T*>(out), state_out);
    return cudaGetLastError();
}

bool chunked_f32_d128_supports(const Problem& p, int dtype, const void* q, const void* k,
                               const void* v, const void* out, const float* state_in,
                               const float* state_out);
cudaError_t launch_chunked_f32_d128(const Problem& p, int dtype, const void* q, const void* k,
                                    const void* v, const float* g, const float* beta,
                                    const float* state_in, void* out, float* state_out,
                                    cudaStream_t stream);

// The CUDA-core chunked path: the register-tiled kernel for d_k = d_v = 128,
// chunk 64 (gdr_chunked_f32.cu) when its vector accesses are aligned, this
// kernel for every other shape.
cudaError_t launch_chunked_ffma(const Problem& p, int dtype, const void* q, const void* k,
                                const void* v, const float* g, const float* beta,
                                const float* state_in, void* out, float* state_out,
                                cudaStream_t stream) {
    if (chunked_f32_d128_supports(p, dtype, q, k, v, out, state_in, state_out))
        return launch_chunked_f32_d128(p, dtype, q, k, v, g, beta, state_in, out, state_out,
                                       stream);
    if (dtype == GDR_DTYPE_BF16)
        return launch_ffma_t<__nv_bfloat16>(p, q, k, v, g, beta, state_in, out, state_out,
                                            stream);
    if (dtype == GDR_DTYPE_F16)
        return launch_ffma_t<__half>(p, q, k, v, g, beta, state_in, out, state_out, stream);
    return launch_ffma_t<float>(p, q, k, v, g, beta, state_in, out, state_out, stream);
}

}  // namespace gdr
