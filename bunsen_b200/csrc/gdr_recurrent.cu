// GatedDeltaRule::recurrent (delta_rule.rs:182-209) on CUDA cores.
//
// Per (sequence, value head) and position t, with S the [d_k, d_v] f32 state:
//   S <- exp(g_t) S;  read = k_t^T S;  delta = (v_t - read) beta_t;
//   S <- S + k_t delta^T;  o_t = q_t^T S
// q_t, k_t L2-normalised (when asked) and q_t scaled by 1/sqrt(d_k).
//
// Two kernels:
//  * recurrent_d128 -- d_k = d_v = 128, the decode hot path. Bandwidth bound:
//    each state is read from HBM once and written once (64 KiB each way per
//    head). One CTA of 256 threads per (sequence, head): warp w holds state
//    rows w, w+8, ..., w+120 and lane l columns 4l..4l+3, in registers, so
//    every state access is a 128-bit load/store and a warp touches one whole
//    512-byte row per instruction. The two reductions over d_k (k^T S and
//    q^T S) run in one pass: o = q^T S_decayed + delta (q . k), which is
//    q^T S after the rank-one update. One smem exchange per position.
//  * recurrent_generic -- any d_k, d_v <= 256: the state in shared memory,
//    one thread per column, in column blocks of one CTA each when the state
//    is large. For small or unusual head sizes (bunsen's unit test shapes);
//    not a performance path.
#include "gdr_common.cuh"
#include "gdr_decode.cuh"

namespace gdr {

namespace {

template <typename T>
__global__ void __launch_bounds__(256, 2)
recurrent_d128(Problem p, const T* __restrict__ q, const T* __restrict__ k,
               const T* __restrict__ v, const float* __restrict__ g,
               const float* __restrict__ beta, const float* state_in, T* __restrict__ out,
               float* state_out) {
    __shared__ __align__(16) uint8_t smem[sizeof(DecodeSmem)];
    const int h = blockIdx.x, s = blockIdx.y;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t hs = (static_cast<int64_t>(s) * p.heads_v + h) * kDecD * kDecD;
    recurrent_d128_item<T>(p, q, k, v, g, beta, t0, t1, h, state_in ? state_in + hs : nullptr,
                           out, state_out + hs, smem);
}

// Any d_k, d_v <= 256. A state's columns evolve independently (column j
// needs only k, q and v[j]), so each CTA takes `cols` of them (grid z) and
// keeps S[:, c0 .. c0 + w) in shared memory, with q and k.
template <typename T>
__global__ void __launch_bounds__(128)
recurrent_generic(Problem p, const T* __restrict__ q, const T* __restrict__ k,
                  const T* __restrict__ v, const float* __restrict__ g,
                  const float* __restrict__ beta, const float* state_in, T* __restrict__ out,
                  float* state_out, int cols) {
    extern __shared__ float smem[];
    const int dk = p.d_k, dv = p.d_v;
    const int c0 = static_cast<int>(blockIdx.z) * cols;
    const int w = dv - c0 < cols ? dv - c0 : cols;  // this CTA's columns
    float* S = smem;                 // [dk][w]
    float* qv = S + dk * cols;       // [dk]
    float* kv = qv + dk;             // [dk]
    __shared__ float norms[2];
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t head_state = (static_cast<int64_t>(s) * p.heads_v + h) * dk * dv + c0;
    for (int e = tid; e < dk * w; e += blockDim.x) {
        const int i = e / w, j = e - i * w;
        S[e] = state_in ? state_in[head_state + static_cast<int64_t>(i) * dv + j] : 0.f;
    }
    const int hq = h / p.group;
    for (int64_t t = t0; t < t1; ++t) {
        const int64_t qk_off = (t * p.heads_qk + hq) * dk;
        for (int i = tid; i < dk; i += blockDim.x) {
            qv[i] = to_f32(q[qk_off + i]);
            kv[i] = to_f32(k[qk_off + i]);
        }
        __syncthreads();
        if (tid < 64) {  // warp 0: |q|^2, warp 1: |k|^2
            const float* x = tid < 32 ? qv : kv;
            float acc = 0.f;
            for (int i = tid & 31; i < dk; i += 32) acc = fmaf(x[i], x[i], acc);
            acc = warp_sum(acc);
            if ((tid & 31) == 0) norms[tid >> 5] = acc;
        }
        __syncthreads();
        const float fq = l2_factor(p, norms[0]) * p.q_scale, fk = l2_factor(p, norms[1]);
        const int64_t gate = t * p.heads_v + h;
        float gt, bt;
        rule_gates(p, g, beta, gate, h, gt, bt);
        const float decay = __expf(gt);
        for (int j = tid; j < w; j += blockDim.x) {
            float read = 0.f;
            for (int i = 0; i < dk; ++i) {
                S[i * w + j] *= decay;
                read = fmaf(kv[i] * fk, S[i * w + j], read);
            }
            const float d = (to_f32(v[(t * p.heads_v + h) * dv + c0 + j]) - read) * bt;
            float o = 0.f;
            for (int i = 0; i < dk; ++i) {
                S[i * w + j] = fmaf(kv[i] * fk, d, S[i * w + j]);
                o = fmaf(qv[i] * fq, S[i * w + j], o);
            }
            out[(t * p.heads_v + h) * dv + c0 + j] = from_f32<T>(o);
        }
        __syncthreads();
    }
    for (int e = tid; e < dk * w; e += blockDim.x) {
        const int i = e / w, j = e - i * w;
        state_out[head_state + static_cast<int64_t>(i) * dv + j] = S[e];
    }
}

// Shared memory of a recurrent_generic (or recurrent_f64) CTA is kept under
// this, so any d_k, d_v <= 256 fits (a 256 x 256 f32 state runs as three
// column blocks, an f64 one as six).
constexpr int kGenericSmemCap = 96 * 1024;

__device__ __forceinline__ double warp_sum_f64(double x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// recurrent_generic in f64, for f64 inputs: bunsen computes in f64 when its
// inputs are f64 (burner/tensor/widening.rs:58-60), g, beta and the state
// included. `eps`: qk_l2norm_eps in f64.
__global__ void __launch_bounds__(128)
recurrent_f64(Problem p, double eps, const double* __restrict__ q, const double* __restrict__ k,
              const double* __restrict__ v, const double* __restrict__ g,
              const double* __restrict__ beta, const double* state_in, double* __restrict__ out,
              double* state_out, int cols) {
    extern __shared__ double smem64[];
    const int dk = p.d_k, dv = p.d_v;
    const int c0 = static_cast<int>(blockIdx.z) * cols;
    const int w = dv - c0 < cols ? dv - c0 : cols;  // this CTA's columns
    double* S = smem64;              // [dk][w]
    double* qv = S + dk * cols;      // [dk]
    double* kv = qv + dk;            // [dk]
    __shared__ double norms[2];
    const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t head_state = (static_cast<int64_t>(s) * p.heads_v + h) * dk * dv + c0;
    for (int e = tid; e < dk * w; e += blockDim.x) {
        const int i = e / w, j = e - i * w;
        S[e] = state_in ? state_in[head_state + static_cast<int64_t>(i) * dv + j] : 0.0;
    }
    const int hq = h / p.group;
    const double q_scale = 1.0 / sqrt(static_cast<double>(dk));
    for (int64_t t = t0; t < t1; ++t) {
        const int64_t qk_off = (t * p.heads_qk + hq) * dk;
        for (int i = tid; i < dk; i += blockDim.x) {
            qv[i] = q[qk_off + i];
            kv[i] = k[qk_off + i];
        }
        __syncthreads();
        if (tid < 64) {  // warp 0: |q|^2, warp 1: |k|^2
            const double* x = tid < 32 ? qv : kv;
            double acc = 0.0;
            for (int i = tid & 31; i < dk; i += 32) acc = fma(x[i], x[i], acc);
            acc = warp_sum_f64(acc);
            if ((tid & 31) == 0) norms[tid >> 5] = acc;
        }
        __syncthreads();
        const double fq = (p.use_l2norm ? 1.0 / sqrt(norms[0] + eps) : 1.0) * q_scale;
        const double fk = p.use_l2norm ? 1.0 / sqrt(norms[1] + eps) : 1.0;
        const int64_t gate = t * p.heads_v + h;
        const double decay = exp(g[gate]), bt = beta[gate];
        for (int j = tid; j < w; j += blockDim.x) {
            double read = 0.0;
            for (int i = 0; i < dk; ++i) {
                S[i * w + j] *= decay;
                read = fma(kv[i] * fk, S[i * w + j], read);
            }
            const double d = (v[(t * p.heads_v + h) * dv + c0 + j] - read) * bt;
            double o = 0.0;
            for (int i = 0; i < dk; ++i) {
                S[i * w + j] = fma(kv[i] * fk, d, S[i * w + j]);
                o = fma(qv[i] * fq, S[i * w + j], o);
            }
            out[(t * p.heads_v + h) * dv + c0 + j] = o;
        }
        __syncthreads();
    }
    for (int e = tid; e < dk * w; e += blockDim.x) {
        const int i = e / w, j = e - i * w;
        state_out[head_state + static_cast<int64_t>(i) * dv + j] = S[e];
    }
}

// Column blocks of equal width for a state of d_k rows of `elem`-byte values,
// each CTA's share (plus q and k) under kGenericSmemCap.
void column_blocks(int d_k, int d_v, int elem, int& blocks, int& cols, size_t& smem) {
    const int max_cols = (kGenericSmemCap - 2 * d_k * elem) / (d_k * elem);
    blocks = (d_v + max_cols - 1) / max_cols;
    cols = (d_v + blocks - 1) / blocks;
    smem = static_cast<size_t>(elem) * (static_cast<size_t>(d_k) * cols + 2 * d_k);
}

}  // namespace

template <typename T>
static cudaError_t launch_recurrent_t(const Problem& p, const void* q, const void* k,
                                      const void* v, const float* g, const float* beta,
                                      const float* state_in, void* out, float* state_out,
                                      cudaStream_t stream) {
    const dim3 grid(p.heads_v, p.n_seqs);
    if (p.d_k == kDecD && p.d_v == kDecD) {
        recurrent_d128<T><<<grid, 256, 0, stream>>>(
            p, static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g,
            beta, state_in, static_cast<T*>(out), state_out);
    } else {
        int blocks, cols;
        size_t smem;
        column_blocks(p.d_k, p.d_v, static_cast<int>(sizeof(float)), blocks, cols, smem);
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(recurrent_generic<T>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
            if (e != cudaSuccess) return e;
        }
        recurrent_generic<T><<<dim3(p.heads_v, p.n_seqs, blocks), 128, smem, stream>>>(
            p, static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g,
            beta, state_in, static_cast<T*>(out), state_out, cols);
    }
    return cudaGetLastError();
}

cudaError_t launch_recurrent(const Problem& p, int dtype, const void* q, const void* k,
                             const void* v, const float* g, const float* beta,
                             const float* state_in, void* out, float* state_out,
                             cudaStream_t stream) {
    if (dtype == GDR_DTYPE_BF16)
        return launch_recurrent_t<__nv_bfloat16>(p, q, k, v, g, beta, state_in, out, state_out,
                                                 stream);
    if (dtype == GDR_DTYPE_F16)
        return launch_recurrent_t<__half>(p, q, k, v, g, beta, state_in, out, state_out, stream);
    return launch_recurrent_t<float>(p, q, k, v, g, beta, state_in, out, state_out, stream);
}

cudaError_t launch_recurrent_f64(const Problem& p, double eps, const double* q, const double* k,
                                 const double* v, const double* g, const double* beta,
                                 const double* state_in, double* out, double* state_out,
                                 cudaStream_t stream) {
    int blocks, cols;
    size_t smem;
    column_blocks(p.d_k, p.d_v, static_cast<int>(sizeof(double)), blocks, cols, smem);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            recurrent_f64, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    recurrent_f64<<<dim3(p.heads_v, p.n_seqs, blocks), 128, smem, stream>>>(
        p, eps, q, k, v, g, beta, state_in, out, state_out, cols);
    return cudaGetLastError();
}

}  // namespace gdr
