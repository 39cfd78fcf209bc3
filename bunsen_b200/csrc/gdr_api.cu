// The extern "C" entry points of include/gdr.h: argument checks (bunsen's
// shape contracts, delta_rule.rs:135-150 and :233, become GDR_ERR_INVALID),
// then the kernel that serves the call.
#include <cmath>
#include <mutex>
#include <vector>

#include "gdr_common.cuh"

namespace gdr {
cudaError_t launch_recurrent(const Problem&, int, const void*, const void*, const void*,
                             const float*, const float*, const float*, void*, float*,
                             cudaStream_t);
cudaError_t launch_chunked_ffma(const Problem&, int, const void*, const void*, const void*,
                                const float*, const float*, const float*, void*, float*,
                                cudaStream_t);
bool chunked_ffma_supports(int dk, int dv, int c);
bool chunked_tc_supports(const gdr_params& p);
cudaError_t launch_chunked_tc(const Problem&, const void*, const void*, const void*,
                              const float*, const float*, const float*, void*, float*,
                              cudaStream_t);
bool split_may_help(const Problem& p);
cudaError_t launch_chunked_split(const Problem&, const void*, const void*, const void*,
                                 const float*, const float*, const float*, void*, float*, int,
                                 cudaStream_t);
cudaError_t launch_recurrent_f64(const Problem& p, double eps, const double* q, const double* k,
                                 const double* v, const double* g, const double* beta,
                                 const double* state_in, double* out, double* state_out,
                                 cudaStream_t stream);
cudaError_t take_device_error(int* flag);
cudaError_t take_layer_error(int* flag);
cudaError_t library_pool(cudaMemPool_t* pool, bool create);
int conv_max_taps();
cudaError_t launch_causal_conv1d(int dtype, int32_t n_seqs, int64_t tokens, int32_t seq_len,
                                 const int32_t* cu_seqlens, int32_t channels, int32_t taps,
                                 int32_t split0, int32_t split1, int32_t silu, const void* x,
                                 const void* weight, const float* state_in, void* out0,
                                 void* out1, void* out2, float* state_out, cudaStream_t s);
cudaError_t launch_gates(int dtype, int64_t n, int heads, const void* a, const void* b,
                         const float* a_log, const float* dt_bias, float* g, float* beta,
                         cudaStream_t s);
cudaError_t launch_gated_norm(int dtype, int64_t rows, int width, const void* x, const void* z,
                              const float* weight, float eps, void* out, cudaStream_t s);
cudaError_t launch_reorder(const void* src, void* dst, const int32_t* sources, int32_t rows,
                           int32_t src_rows, size_t row_bytes, cudaStream_t s);
cudaError_t launch_selftest_wait(uint64_t limit_ns, cudaStream_t stream);
int mixed_noalloc_max_seqs();
cudaError_t launch_mixed_tc_noalloc(const Problem&, const void*, const void*, const void*,
                                    const float*, const float*, float*, const int32_t*, int32_t,
                                    void*, cudaStream_t);
size_t mixed_workspace_bytes(int n_seqs);
cudaError_t launch_mixed_tc(const Problem&, const void*, const void*, const void*, const float*,
                            const float*, float*, const int32_t*, int32_t, void*, int32_t*,
                            cudaStream_t);
}  // namespace gdr

namespace {

using gdr::Problem;

int64_t total_tokens(const Problem& p) {
    return p.cu_seqlens ? p.seq_len : static_cast<int64_t>(p.n_seqs) * p.seq_len;
}

// Checks what the host can check and fills the kernels' descriptor. `f64`:
// the call is one of the f64 entry points, whose dtype is GDR_DTYPE_F64.
gdr_status make_problem(const gdr_params* params, const int32_t* cu_seqlens, Problem& p,
                        bool f64 = false) {
    if (params == nullptr) return GDR_ERR_INVALID;
    const gdr_params& a = *params;
    if (a.heads_qk <= 0 || a.heads_v <= 0 || a.heads_v % a.heads_qk != 0) return GDR_ERR_INVALID;
    if (a.d_k <= 0 || a.d_v <= 0 || a.seq_len < 0) return GDR_ERR_INVALID;
    if (f64 ? a.dtype != GDR_DTYPE_F64
            : (a.dtype != GDR_DTYPE_F32 && a.dtype != GDR_DTYPE_BF16 && a.dtype != GDR_DTYPE_F16))
        return GDR_ERR_INVALID;
    if (a.use_l2norm && !(a.l2norm_eps >= 0.0)) return GDR_ERR_INVALID;
    if (cu_seqlens == nullptr && a.batch < 0) return GDR_ERR_INVALID;
    if (cu_seqlens != nullptr && a.n_seqs < 0) return GDR_ERR_INVALID;
    p.n_seqs = cu_seqlens ? a.n_seqs : a.batch;
    p.seq_len = a.seq_len;
    p.cu_seqlens = cu_seqlens;
    p.heads_qk = a.heads_qk;
    p.heads_v = a.heads_v;
    p.group = a.heads_v / a.heads_qk;
    p.d_k = a.d_k;
    p.d_v = a.d_v;
    p.chunk = a.chunk_size;
    p.use_l2norm = a.use_l2norm != 0;
    p.l2norm_eps = static_cast<float>(a.l2norm_eps);
    p.q_scale = 1.0f / std::sqrt(static_cast<float>(a.d_k));
    if (p.n_seqs > 65535 || p.heads_v > 65535) return GDR_ERR_UNSUPPORTED;  // grid limits
    return GDR_OK;
}

// Token buffers may be NULL only when there are no tokens (an empty tensor
// has no storage); the state is written whenever there are sequences.
bool io_ok(const Problem& p, const void* q, const void* k, const void* v, const void* g,
           const void* beta, const void* out, const void* state_out) {
    const bool tokens = total_tokens(p) > 0;
    return (!tokens || (q && k && v && g && beta && out)) && (p.n_seqs == 0 || state_out);
}

gdr_status from_cuda(cudaError_t e) { return e == cudaSuccess ? GDR_OK : GDR_ERR_CUDA; }

enum class ChunkedPath { kNothing, kPassThrough, kTensor, kSplit, kCudaCore, kRecurrent };

// The recurrent kernels' head sizes.
constexpr int kRecurrentMaxD = 256;

// Which kernels a gdr_chunked call runs: the checks of everything but the
// buffers, then the algorithm (GDR_ALGO_AUTO: the tensor-core kernels where
// they apply -- split into segments when that may help -- else the f32
// chunked kernel, else, for chunks above 64 or heads above 128, the recurrent
// kernel: the same rule, delta_rule.rs:549-608).
gdr_status chunked_path(const gdr_params* params, const int32_t* cu_seqlens, Problem& p,
                        ChunkedPath& path) {
    gdr_status st = make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    if (params->chunk_size <= 0) return GDR_ERR_INVALID;  // delta_rule.rs:233
    const int algo = params->algo;
    if (algo != GDR_ALGO_AUTO && algo != GDR_ALGO_CUDA_CORE && algo != GDR_ALGO_TENSOR &&
        algo != GDR_ALGO_TENSOR_SPLIT)
        return GDR_ERR_INVALID;
    if (params->split_chunks < 0) return GDR_ERR_INVALID;
    const bool tc_ok = gdr::chunked_tc_supports(*params);
    const bool ffma_ok = gdr::chunked_ffma_supports(p.d_k, p.d_v, p.chunk);
    const bool rec_ok = p.d_k <= kRecurrentMaxD && p.d_v <= kRecurrentMaxD;
    if (algo == GDR_ALGO_TENSOR || algo == GDR_ALGO_TENSOR_SPLIT) {
        if (!tc_ok) return GDR_ERR_UNSUPPORTED;
        path = algo == GDR_ALGO_TENSOR ? ChunkedPath::kTensor : ChunkedPath::kSplit;
    } else if (algo == GDR_ALGO_CUDA_CORE) {
        if (!ffma_ok && !rec_ok) return GDR_ERR_UNSUPPORTED;
        path = ffma_ok ? ChunkedPath::kCudaCore : ChunkedPath::kRecurrent;
    } else {
        if (!tc_ok && !ffma_ok && !rec_ok) return GDR_ERR_UNSUPPORTED;
        path = tc_ok ? ((params->split_chunks > 0 || gdr::split_may_help(p)) ? ChunkedPath::kSplit
                                                                             : ChunkedPath::kTensor)
               : ffma_ok ? ChunkedPath::kCudaCore
                         : ChunkedPath::kRecurrent;
    }
    if (p.n_seqs == 0) path = ChunkedPath::kNothing;
    else if (total_tokens(p) == 0) path = ChunkedPath::kPassThrough;
    return GDR_OK;
}

// ---- host-buffer calls ----------------------------------------------------
constexpr int kHostStreams = 3;  // groups in flight: copy in, run, copy out
#ifndef GDR_HOST_GROUPS
#define GDR_HOST_GROUPS 16
#endif
constexpr int kHostGroups = GDR_HOST_GROUPS;  // groups of whole sequences per call

// The worker streams of gdr_chunked_host, created once per device and kept.
cudaError_t host_streams(cudaStream_t** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static cudaStream_t streams[kMaxDevices][kHostStreams] = {};
    static bool made[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!made[dev]) {
        for (int i = 0; i < kHostStreams; ++i)
            if ((e = cudaStreamCreateWithFlags(&streams[dev][i], cudaStreamNonBlocking)) !=
                cudaSuccess) {
                while (i-- > 0) cudaStreamDestroy(streams[dev][i]);  // next call starts over
                return e;
            }
        made[dev] = true;
    }
    *out = streams[dev];
    return cudaSuccess;
}

// A group's cu_seqlens, counted from its first token.
__global__ void rebase_offsets(const int32_t* cu, int32_t n1, int32_t* out) {
    const int32_t base = cu[0];
    for (int i = threadIdx.x; i < n1; i += blockDim.x) out[i] = cu[i] - base;
}

}  // namespace

extern "C" {

gdr_status gdr_recurrent(const gdr_params* params, const void* q, const void* k, const void* v,
                         const float* g, const float* beta, const float* state_in, void* out,
                         float* state_out, const int32_t* cu_seqlens, void* stream) {
    Problem p;
    gdr_status st = make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    if (!io_ok(p, q, k, v, g, beta, out, state_out)) return GDR_ERR_INVALID;
    if (p.d_k > kRecurrentMaxD || p.d_v > kRecurrentMaxD) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0) return GDR_OK;
    return from_cuda(gdr::launch_recurrent(p, params->dtype, q, k, v, g, beta, state_in, out,
                                           state_out, static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_recurrent_f64(const gdr_params* params, const double* q, const double* k,
                             const double* v, const double* g, const double* beta,
                             const double* state_in, double* out, double* state_out,
                             const int32_t* cu_seqlens, void* stream) {
    Problem p;
    gdr_status st = make_problem(params, cu_seqlens, p, true);
    if (st != GDR_OK) return st;
    if (!io_ok(p, q, k, v, g, beta, out, state_out)) return GDR_ERR_INVALID;
    if (p.d_k > kRecurrentMaxD || p.d_v > kRecurrentMaxD) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0) return GDR_OK;
    return from_cuda(gdr::launch_recurrent_f64(p, params->l2norm_eps, q, k, v, g, beta, state_in,
                                               out, state_out,
                                               static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_chunked_f64(const gdr_params* params, const double* q, const double* k,
                           const double* v, const double* g, const double* beta,
                           const double* state_in, double* out, double* state_out,
                           const int32_t* cu_seqlens, void* stream) {
    if (params != nullptr && params->chunk_size <= 0) return GDR_ERR_INVALID;  // delta_rule.rs:233
    return gdr_recurrent_f64(params, q, k, v, g, beta, state_in, out, state_out, cu_seqlens,
                             stream);
}

gdr_status gdr_chunked(const gdr_params* params, const void* q, const void* k, const void* v,
                       const float* g, const float* beta, const float* state_in, void* out,
                       float* state_out, const int32_t* cu_seqlens, void* stream) {
    Problem p;
    ChunkedPath path;
    gdr_status st = chunked_path(params, cu_seqlens, p, path);
    if (st != GDR_OK) return st;
    if (!io_ok(p, q, k, v, g, beta, out, state_out)) return GDR_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (path) {
        case ChunkedPath::kNothing:
            return GDR_OK;
        case ChunkedPath::kPassThrough:  // no tokens: the state passes through
        case ChunkedPath::kRecurrent:
            return from_cuda(gdr::launch_recurrent(p, params->dtype, q, k, v, g, beta, state_in,
                                                   out, state_out, s));
        case ChunkedPath::kSplit:
            return from_cuda(gdr::launch_chunked_split(p, q, k, v, g, beta, state_in, out,
                                                       state_out, params->split_chunks, s));
        case ChunkedPath::kTensor:
            return from_cuda(
                gdr::launch_chunked_tc(p, q, k, v, g, beta, state_in, out, state_out, s));
        case ChunkedPath::kCudaCore:
            break;
    }
    return from_cuda(gdr::launch_chunked_ffma(p, params->dtype, q, k, v, g, beta, state_in, out,
                                              state_out, s));
}

int32_t gdr_chunked_launches(const gdr_params* params, int32_t packed) {
    const int32_t any = 0;  // stands for a cu_seqlens pointer; never read
    Problem p;
    ChunkedPath path;
    if (chunked_path(params, packed ? &any : nullptr, p, path) != GDR_OK) return -1;
    switch (path) {
        case ChunkedPath::kNothing: return 0;
        case ChunkedPath::kSplit: return 4;  // plan, pass A, scan, pass B
        default: return 1;
    }
}

gdr_status gdr_chunked_host(const gdr_params* params, const void* q, const void* k,
                            const void* v, const float* g, const float* beta,
                            const float* state_in, void* out, float* state_out,
                            const int32_t* cu_seqlens, void* stream) {
    Problem p;
    ChunkedPath path;
    gdr_status st = chunked_path(params, cu_seqlens, p, path);
    if (st != GDR_OK) return st;
    if (!io_ok(p, q, k, v, g, beta, out, state_out)) return GDR_ERR_INVALID;
    if (path == ChunkedPath::kNothing) return GDR_OK;
    const bool packed = cu_seqlens != nullptr;
    const int n = p.n_seqs;
    const int64_t total = total_tokens(p);
    // Sequence s covers tokens [first(s), first(s + 1)).
    if (packed) {
        if (cu_seqlens[0] != 0 || cu_seqlens[n] != total) return GDR_ERR_INVALID;
        for (int s = 0; s < n; ++s)
            if (cu_seqlens[s + 1] < cu_seqlens[s]) return GDR_ERR_INVALID;
    }
    auto first = [&](int s) -> int64_t {
        return packed ? cu_seqlens[s] : static_cast<int64_t>(s) * p.seq_len;
    };
    // Groups of whole sequences of about total / kHostGroups tokens each.
    std::vector<int> cut{0};
    const int64_t want = (total + kHostGroups - 1) / kHostGroups;
    for (int s = 1; s < n; ++s)
        if (first(s) - first(cut.back()) >= want) cut.push_back(s);
    cut.push_back(n);
    const int groups = static_cast<int>(cut.size()) - 1;
    int64_t max_tok = 0, max_seq = 0;
    for (int i = 0; i < groups; ++i) {
        max_tok = std::max<int64_t>(max_tok, first(cut[i + 1]) - first(cut[i]));
        max_seq = std::max<int64_t>(max_seq, cut[i + 1] - cut[i]);
    }
    const size_t es = params->dtype == GDR_DTYPE_F32 ? 4 : 2;
    const size_t row_qk = static_cast<size_t>(p.heads_qk) * p.d_k * es;
    const size_t row_v = static_cast<size_t>(p.heads_v) * p.d_v * es;
    const size_t row_gb = static_cast<size_t>(p.heads_v) * sizeof(float);
    const size_t one_state = static_cast<size_t>(p.heads_v) * p.d_k * p.d_v * sizeof(float);
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    // One slot of device buffers per worker stream.
    const size_t o_q = 0, o_k = o_q + up(max_tok * row_qk), o_v = o_k + up(max_tok * row_qk),
                 o_o = o_v + up(max_tok * row_v), o_g = o_o + up(max_tok * row_v),
                 o_b = o_g + up(max_tok * row_gb), o_s = o_b + up(max_tok * row_gb),
                 o_c = o_s + up(max_seq * one_state), slot = o_c + up((max_seq + 1) * 4);
    const size_t o_all = kHostStreams * slot;
    const size_t bytes = o_all + up((static_cast<size_t>(n) + 1) * 4);

    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    cudaStream_t* ws = nullptr;
    cudaMemPool_t pool;
    cudaError_t e = host_streams(&ws);
    if (e == cudaSuccess) e = gdr::library_pool(&pool, true);
    void* mem = nullptr;
    if (e == cudaSuccess) e = cudaMallocFromPoolAsync(&mem, bytes, pool, caller);
    if (e != cudaSuccess) return GDR_ERR_CUDA;
    uint8_t* base = static_cast<uint8_t*>(mem);
    int32_t* cu_all = reinterpret_cast<int32_t*>(base + o_all);
    // Each CUDA call below runs only while every earlier one succeeded.
#define GDR_TRY(call)                      \
    do {                                   \
        if (e == cudaSuccess) e = (call);  \
    } while (0)
    if (packed)
        GDR_TRY(cudaMemcpyAsync(cu_all, cu_seqlens, (static_cast<size_t>(n) + 1) * 4,
                                cudaMemcpyHostToDevice, caller));
    cudaEvent_t start = nullptr, done[kHostStreams] = {};
    GDR_TRY(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
    for (int w = 0; w < kHostStreams; ++w)
        GDR_TRY(cudaEventCreateWithFlags(&done[w], cudaEventDisableTiming));
    GDR_TRY(cudaEventRecord(start, caller));
    for (int w = 0; w < kHostStreams; ++w) GDR_TRY(cudaStreamWaitEvent(ws[w], start, 0));
    auto h2d = [&](void* dst, const void* src, size_t len, cudaStream_t s) {
        if (len > 0) GDR_TRY(cudaMemcpyAsync(dst, src, len, cudaMemcpyHostToDevice, s));
    };
    auto d2h = [&](void* dst, const void* src, size_t len, cudaStream_t s) {
        if (len > 0) GDR_TRY(cudaMemcpyAsync(dst, src, len, cudaMemcpyDeviceToHost, s));
    };
    const auto* hq = static_cast<const uint8_t*>(q);
    const auto* hk = static_cast<const uint8_t*>(k);
    const auto* hv = static_cast<const uint8_t*>(v);
    auto* ho = static_cast<uint8_t*>(out);
    for (int i = 0; i < groups && e == cudaSuccess; ++i) {
        const int w = i % kHostStreams;
        cudaStream_t s = ws[w];
        uint8_t* b = base + w * slot;
        const int s0 = cut[i], ns = cut[i + 1] - cut[i];
        const int64_t t0 = first(s0), nt = first(cut[i + 1]) - t0;
        h2d(b + o_q, hq + t0 * row_qk, nt * row_qk, s);
        h2d(b + o_k, hk + t0 * row_qk, nt * row_qk, s);
        h2d(b + o_v, hv + t0 * row_v, nt * row_v, s);
        h2d(b + o_g, g + t0 * p.heads_v, nt * row_gb, s);
        h2d(b + o_b, beta + t0 * p.heads_v, nt * row_gb, s);
        if (state_in) h2d(b + o_s, state_in + s0 * (one_state / 4), ns * one_state, s);
        int32_t* cu = reinterpret_cast<int32_t*>(b + o_c);
        if (packed && e == cudaSuccess) {
            rebase_offsets<<<1, 256, 0, s>>>(cu_all + s0, ns + 1, cu);
            GDR_TRY(cudaGetLastError());
        }
        gdr_params gp = *params;
        if (packed) {
            gp.n_seqs = ns;
            gp.seq_len = static_cast<int32_t>(nt);
        } else {
            gp.batch = ns;
        }
        float* ds = reinterpret_cast<float*>(b + o_s);
        const gdr_status r =
            gdr_chunked(&gp, b + o_q, b + o_k, b + o_v, reinterpret_cast<float*>(b + o_g),
                        reinterpret_cast<float*>(b + o_b), state_in ? ds : nullptr, b + o_o, ds,
                        packed ? cu : nullptr, s);
        if (r != GDR_OK && e == cudaSuccess) e = cudaErrorLaunchFailure;
        d2h(ho + t0 * row_v, b + o_o, nt * row_v, s);
        d2h(state_out + s0 * (one_state / 4), ds, ns * one_state, s);
    }
#undef GDR_TRY
    // The caller's stream waits for every worker; the scratch is freed after.
    // Where that order could not be set up (an earlier failure), the workers
    // are drained on the host first, so no copy still in flight can touch the
    // scratch once the pool hands it out again.
    bool ordered = true;
    for (int w = 0; w < kHostStreams; ++w) {
        cudaError_t r = done[w] != nullptr ? cudaEventRecord(done[w], ws[w])
                                           : cudaErrorInvalidResourceHandle;
        if (r == cudaSuccess) r = cudaStreamWaitEvent(caller, done[w], 0);
        if (r != cudaSuccess) {
            ordered = false;
            if (e == cudaSuccess) e = r;
        }
    }
    if (!ordered)
        for (int w = 0; w < kHostStreams; ++w) cudaStreamSynchronize(ws[w]);
    const cudaError_t f = cudaFreeAsync(mem, caller);
    if (start != nullptr) cudaEventDestroy(start);
    for (int w = 0; w < kHostStreams; ++w)
        if (done[w] != nullptr) cudaEventDestroy(done[w]);
    return from_cuda(e != cudaSuccess ? e : f);
}

gdr_status gdr_causal_conv1d(const gdr_conv_params* params, const void* x, const void* weight,
                             const float* state_in, void* out0, void* out1, void* out2,
                             float* state_out, const int32_t* cu_seqlens, void* stream) {
    if (params == nullptr) return GDR_ERR_INVALID;
    const gdr_conv_params& a = *params;
    const int C = a.channels, K = a.taps;
    if (C <= 0 || K < 2 || a.seq_len < 0) return GDR_ERR_INVALID;  // causal_conv.rs:47
    if (K > gdr::conv_max_taps()) return GDR_ERR_UNSUPPORTED;
    if (a.dtype != GDR_DTYPE_F32 && a.dtype != GDR_DTYPE_BF16 && a.dtype != GDR_DTYPE_F16)
        return GDR_ERR_INVALID;
    if (!(0 <= a.split0 && a.split0 <= a.split1 && a.split1 <= C)) return GDR_ERR_INVALID;
    const int32_t n = cu_seqlens ? a.n_seqs : a.batch;
    if (n < 0) return GDR_ERR_INVALID;
    const int64_t tokens = cu_seqlens ? a.seq_len : static_cast<int64_t>(a.batch) * a.seq_len;
    if (tokens > 0) {
        if (x == nullptr || weight == nullptr) return GDR_ERR_INVALID;
        if ((a.split0 > 0 && out0 == nullptr) || (a.split1 > a.split0 && out1 == nullptr) ||
            (C > a.split1 && out2 == nullptr))
            return GDR_ERR_INVALID;
    }
    if (n == 0) return GDR_OK;
    return from_cuda(gdr::launch_causal_conv1d(
        a.dtype, n, tokens, a.seq_len, cu_seqlens, C, K, a.split0, a.split1, a.silu != 0, x,
        weight, state_in, out0, out1, out2, state_out, static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_gated_norm(int64_t rows, int32_t width, const void* x, const void* z,
                          const float* weight, double eps, int32_t dtype, void* out,
                          void* stream) {
    if (rows < 0 || width <= 0 || !(eps >= 0.0)) return GDR_ERR_INVALID;
    if (dtype != GDR_DTYPE_F32 && dtype != GDR_DTYPE_BF16 && dtype != GDR_DTYPE_F16)
        return GDR_ERR_INVALID;
    if (rows == 0) return GDR_OK;
    if (x == nullptr || z == nullptr || weight == nullptr || out == nullptr) return GDR_ERR_INVALID;
    return from_cuda(gdr::launch_gated_norm(dtype, rows, width, x, z, weight,
                                            static_cast<float>(eps), out,
                                            static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_state_reorder(const void* src, void* dst, const int32_t* sources, int32_t rows,
                             int32_t src_rows, size_t row_bytes, void* stream) {
    if (rows < 0 || src_rows < 0 || row_bytes % 4 != 0) return GDR_ERR_INVALID;
    if (rows == 0 || row_bytes == 0) return GDR_OK;
    if (src == nullptr || dst == nullptr || sources == nullptr) return GDR_ERR_INVALID;
    const auto* s0 = static_cast<const uint8_t*>(src);
    const auto* d0 = static_cast<const uint8_t*>(dst);
    const size_t sb = static_cast<size_t>(src_rows) * row_bytes,
                 db = static_cast<size_t>(rows) * row_bytes;
    if (d0 < s0 + sb && s0 < d0 + db) return GDR_ERR_INVALID;  // overlap
    return from_cuda(gdr::launch_reorder(src, dst, sources, rows, src_rows, row_bytes,
                                         static_cast<cudaStream_t>(stream)));
}

namespace {

// The checks of a gdr_layer_io every layer call shares (the buffers' own
// alignment needs are the caller's): gates need g and beta absent and their
// four inputs, the norm its weight and a non-negative epsilon.
gdr_status check_layer_io(const gdr_layer_io& io, int64_t tokens, const float* g,
                          const float* beta) {
    if (io.gate_a != nullptr) {
        if (g != nullptr || beta != nullptr) return GDR_ERR_INVALID;
        if (io.gate_dtype != GDR_DTYPE_F32 && io.gate_dtype != GDR_DTYPE_BF16 &&
            io.gate_dtype != GDR_DTYPE_F16)
            return GDR_ERR_INVALID;
        if (tokens > 0 && (io.gate_b == nullptr || io.a_log == nullptr || io.dt_bias == nullptr))
            return GDR_ERR_INVALID;
    }
    if (io.norm_z != nullptr &&
        ((tokens > 0 && io.norm_weight == nullptr) || !(io.norm_eps >= 0.0)))
        return GDR_ERR_INVALID;
    return GDR_OK;
}

// The fused steps' inputs into the kernels' descriptor.
void set_layer_gates(const gdr_layer_io& io, Problem& p) {
    p.gate_a = io.gate_a;
    p.gate_b = io.gate_b;
    p.a_log = io.a_log;
    p.dt_bias = io.dt_bias;
    p.gate_dtype = io.gate_dtype;
    p.gate_bf16 = io.gate_dtype == GDR_DTYPE_BF16;
}
void set_layer_norm(const gdr_layer_io& io, Problem& p) {
    p.norm_z = io.norm_z;
    p.norm_w = io.norm_weight;
    p.norm_eps = static_cast<float>(io.norm_eps);
}

// A rule call with the layer's gates and gated norm. The tensor-core prefill
// (single pass or split) and the recurrent kernels produce g and beta from
// the projections as they stage them, and the tensor-core prefill and the
// d-128 decode apply the norm as they store the output; on the other paths
// the gates are computed first (into stream-ordered scratch from the library
// pool) and the norm is applied to the output after the rule.
gdr_status layer_call(bool chunked, const gdr_params* params, const void* q, const void* k,
                      const void* v, const float* g, const float* beta, const gdr_layer_io* io,
                      const float* state_in, void* out, float* state_out,
                      const int32_t* cu_seqlens, void* stream) {
    auto rule = chunked ? gdr_chunked : gdr_recurrent;
    if (io == nullptr || (io->gate_a == nullptr && io->norm_z == nullptr))
        return rule(params, q, k, v, g, beta, state_in, out, state_out, cu_seqlens, stream);
    Problem p;
    ChunkedPath path = ChunkedPath::kTensor;
    gdr_status st = chunked ? chunked_path(params, cu_seqlens, p, path)
                            : make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    const int64_t tokens = total_tokens(p);
    const bool gates = io->gate_a != nullptr, norm = io->norm_z != nullptr;
    if ((st = check_layer_io(*io, tokens, g, beta)) != GDR_OK) return st;
    const float* g_chk = gates ? static_cast<const float*>(io->gate_a) : g;
    const float* b_chk = gates ? static_cast<const float*>(io->gate_b) : beta;
    if (!io_ok(p, q, k, v, g_chk, b_chk, out, state_out)) return GDR_ERR_INVALID;
    if (!chunked && (p.d_k > 256 || p.d_v > 256)) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0 || (chunked && path == ChunkedPath::kNothing)) return GDR_OK;
    const bool tc = chunked && (path == ChunkedPath::kTensor || path == ChunkedPath::kSplit);
    const bool rec = !chunked || path == ChunkedPath::kRecurrent;  // the recurrent kernels
    const bool d128 = p.d_k == 128 && p.d_v == 128;
    // The tensor-core prefill stages f32 or bf16 projections; the recurrent
    // kernels read any gate dtype.
    const bool fuse_gates = gates && ((tc && io->gate_dtype != GDR_DTYPE_F16) || rec);
    const bool fuse_norm = norm && (tc || (rec && d128));
    // The tensor-core prefill stages 4-byte words of the projections and
    // reads z 16 bytes at a time.
    if (tc && fuse_gates &&
        ((reinterpret_cast<uintptr_t>(io->gate_a) | reinterpret_cast<uintptr_t>(io->gate_b)) & 3))
        return GDR_ERR_INVALID;
    if (tc && fuse_norm && (reinterpret_cast<uintptr_t>(io->norm_z) & 15)) return GDR_ERR_INVALID;
    if (fuse_gates) set_layer_gates(*io, p);
    if (fuse_norm) set_layer_norm(*io, p);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* scratch = nullptr;
    const size_t gates_n = static_cast<size_t>(tokens) * p.heads_v;
    if (gates && !fuse_gates && gates_n > 0) {
        cudaMemPool_t pool;
        if (gdr::library_pool(&pool, true) != cudaSuccess ||
            cudaMallocFromPoolAsync(&scratch, 2 * gates_n * sizeof(float), pool, s) != cudaSuccess)
            return GDR_ERR_CUDA;
        g = static_cast<const float*>(scratch);
        beta = static_cast<const float*>(scratch) + gates_n;
        if (gdr::launch_gates(io->gate_dtype, static_cast<int64_t>(gates_n), p.heads_v, io->gate_a,
                              io->gate_b, io->a_log, io->dt_bias, static_cast<float*>(scratch),
                              static_cast<float*>(scratch) + gates_n, s) != cudaSuccess)
            st = GDR_ERR_CUDA;
    }
    if (st == GDR_OK) {
        cudaError_t e;
        if (rec || path == ChunkedPath::kPassThrough)
            e = gdr::launch_recurrent(p, params->dtype, q, k, v, g, beta, state_in, out, state_out,
                                      s);
        else if (path == ChunkedPath::kSplit)
            e = gdr::launch_chunked_split(p, q, k, v, g, beta, state_in, out, state_out,
                                          params->split_chunks, s);
        else if (path == ChunkedPath::kTensor)
            e = gdr::launch_chunked_tc(p, q, k, v, g, beta, state_in, out, state_out, s);
        else
            e = gdr::launch_chunked_ffma(p, params->dtype, q, k, v, g, beta, state_in, out,
                                         state_out, s);
        st = from_cuda(e);
    }
    if (st == GDR_OK && norm && !fuse_norm && tokens > 0 &&
        gdr::launch_gated_norm(params->dtype, tokens * p.heads_v, p.d_v, out, io->norm_z,
                               io->norm_weight, static_cast<float>(io->norm_eps), out,
                               s) != cudaSuccess)
        st = GDR_ERR_CUDA;
    if (scratch != nullptr && cudaFreeAsync(scratch, s) != cudaSuccess && st == GDR_OK)
        st = GDR_ERR_CUDA;
    return st;
}

}  // namespace

gdr_status gdr_chunked_layer(const gdr_params* params, const void* q, const void* k,
                             const void* v, const float* g, const float* beta,
                             const gdr_layer_io* io, const float* state_in, void* out,
                             float* state_out, const int32_t* cu_seqlens, void* stream) {
    return layer_call(true, params, q, k, v, g, beta, io, state_in, out, state_out, cu_seqlens,
                      stream);
}

gdr_status gdr_recurrent_layer(const gdr_params* params, const void* q, const void* k,
                               const void* v, const float* g, const float* beta,
                               const gdr_layer_io* io, const float* state_in, void* out,
                               float* state_out, const int32_t* cu_seqlens, void* stream) {
    return layer_call(false, params, q, k, v, g, beta, io, state_in, out, state_out, cu_seqlens,
                      stream);
}

size_t gdr_mixed_workspace_size(const gdr_params* params) {
    if (params == nullptr || params->n_seqs < 0) return 0;
    return gdr::mixed_workspace_bytes(params->n_seqs);
}

gdr_status gdr_mixed(const gdr_params* params, const void* q, const void* k, const void* v,
                     const float* g, const float* beta, float* state_pool,
                     const int32_t* state_slots, int32_t n_slots, void* out,
                     const int32_t* cu_seqlens, void* workspace, size_t workspace_bytes,
                     void* stream) {
    if (cu_seqlens == nullptr) return GDR_ERR_INVALID;
    Problem p;
    gdr_status st = make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    if (params->chunk_size <= 0) return GDR_ERR_INVALID;
    if (!io_ok(p, q, k, v, g, beta, out, state_pool)) return GDR_ERR_INVALID;
    if (p.n_seqs > 0 && n_slots <= 0) return GDR_ERR_INVALID;
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 3) != 0 ||
        workspace_bytes < gdr::mixed_workspace_bytes(p.n_seqs))
        return GDR_ERR_INVALID;
    if (!gdr::chunked_tc_supports(*params)) return GDR_ERR_UNSUPPORTED;
    if (static_cast<int64_t>(p.n_seqs) * p.heads_v >= (int64_t{1} << 30)) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0 || total_tokens(p) == 0) return GDR_OK;
    return from_cuda(gdr::launch_mixed_tc(p, q, k, v, g, beta, state_pool, state_slots, n_slots,
                                          out, static_cast<int32_t*>(workspace),
                                          static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_mixed_layer(const gdr_params* params, const void* q, const void* k,
                           const void* v, const float* g, const float* beta,
                           const gdr_layer_io* io, float* state_pool,
                           const int32_t* state_slots, int32_t n_slots, void* out,
                           const int32_t* cu_seqlens, void* workspace, size_t workspace_bytes,
                           void* stream) {
    if (io == nullptr || (io->gate_a == nullptr && io->norm_z == nullptr))
        return gdr_mixed(params, q, k, v, g, beta, state_pool, state_slots, n_slots, out,
                         cu_seqlens, workspace, workspace_bytes, stream);
    if (cu_seqlens == nullptr) return GDR_ERR_INVALID;
    Problem p;
    gdr_status st = make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    if (params->chunk_size <= 0) return GDR_ERR_INVALID;
    const int64_t tokens = total_tokens(p);
    const bool gates = io->gate_a != nullptr, norm = io->norm_z != nullptr;
    if ((st = check_layer_io(*io, tokens, g, beta)) != GDR_OK) return st;
    // The prefill segments stage 4-byte words of the projections and read z
    // 16 bytes at a time.
    if (gates &&
        ((reinterpret_cast<uintptr_t>(io->gate_a) | reinterpret_cast<uintptr_t>(io->gate_b)) & 3))
        return GDR_ERR_INVALID;
    if (norm && (reinterpret_cast<uintptr_t>(io->norm_z) & 15)) return GDR_ERR_INVALID;
    const float* g_chk = gates ? static_cast<const float*>(io->gate_a) : g;
    const float* b_chk = gates ? static_cast<const float*>(io->gate_b) : beta;
    if (!io_ok(p, q, k, v, g_chk, b_chk, out, state_pool)) return GDR_ERR_INVALID;
    if (p.n_seqs > 0 && n_slots <= 0) return GDR_ERR_INVALID;
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 3) != 0 ||
        workspace_bytes < gdr::mixed_workspace_bytes(p.n_seqs))
        return GDR_ERR_INVALID;
    if (!gdr::chunked_tc_supports(*params)) return GDR_ERR_UNSUPPORTED;
    if (static_cast<int64_t>(p.n_seqs) * p.heads_v >= (int64_t{1} << 30)) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0 || tokens == 0) return GDR_OK;
    if (gates) set_layer_gates(*io, p);
    if (norm) set_layer_norm(*io, p);
    return from_cuda(gdr::launch_mixed_tc(p, q, k, v, g, beta, state_pool, state_slots, n_slots,
                                          out, static_cast<int32_t*>(workspace),
                                          static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_mixed_noalloc(const gdr_params* params, const void* q, const void* k,
                             const void* v, const float* g, const float* beta, float* state_pool,
                             const int32_t* state_slots, int32_t n_slots, void* out,
                             const int32_t* cu_seqlens, void* stream) {
    if (cu_seqlens == nullptr) return GDR_ERR_INVALID;
    Problem p;
    gdr_status st = make_problem(params, cu_seqlens, p);
    if (st != GDR_OK) return st;
    if (params->chunk_size <= 0) return GDR_ERR_INVALID;
    if (!io_ok(p, q, k, v, g, beta, out, state_pool)) return GDR_ERR_INVALID;
    if (p.n_seqs > 0 && n_slots <= 0) return GDR_ERR_INVALID;
    if (p.n_seqs > gdr::mixed_noalloc_max_seqs()) return GDR_ERR_CAPACITY;
    if (!gdr::chunked_tc_supports(*params)) return GDR_ERR_UNSUPPORTED;
    if (static_cast<int64_t>(p.n_seqs) * p.heads_v >= (int64_t{1} << 30)) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0 || total_tokens(p) == 0) return GDR_OK;
    return from_cuda(gdr::launch_mixed_tc_noalloc(p, q, k, v, g, beta, state_pool, state_slots,
                                                  n_slots, out, static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_selftest_wait_timeout(int64_t limit_ns, void* stream) {
    if (limit_ns <= 0 || limit_ns > 100000000) return GDR_ERR_INVALID;  // at most 0.1 s
    return from_cuda(gdr::launch_selftest_wait(static_cast<uint64_t>(limit_ns),
                                               static_cast<cudaStream_t>(stream)));
}

gdr_status gdr_device_error(void) {
    int flag = 0, layer = 0;
    if (gdr::take_device_error(&flag) != cudaSuccess) return GDR_ERR_CUDA;
    if (gdr::take_layer_error(&layer) != cudaSuccess) return GDR_ERR_CUDA;
    flag |= layer;
    if (flag & 1) return GDR_ERR_TIMEOUT;
    return (flag & 2) ? GDR_ERR_INVALID : GDR_OK;
}

gdr_status gdr_release_scratch(void) {
    cudaMemPool_t pool = nullptr;
    if (gdr::library_pool(&pool, false) != cudaSuccess) return GDR_ERR_CUDA;
    if (pool == nullptr) return GDR_OK;  // nothing was ever taken on this device
    if (cudaDeviceSynchronize() != cudaSuccess) return GDR_ERR_CUDA;
    return from_cuda(cudaMemPoolTrimTo(pool, 0));
}

const char* gdr_status_string(gdr_status status) {
    switch (status) {
        case GDR_OK: return "ok";
        case GDR_ERR_INVALID: return "invalid argument (shape, pointer or option)";
        case GDR_ERR_UNSUPPORTED: return "no kernel for these dimensions or dtypes";
        case GDR_ERR_CUDA: return "a CUDA call or launch failed";
        case GDR_ERR_TIMEOUT: return "a bounded device-side wait ran out";
        case GDR_ERR_CAPACITY:
            return "more sequences than gdr_mixed_noalloc's fixed work list holds "
                   "(GDR_MIXED_NOALLOC_MAX_SEQS)";
    }
    return "unknown status";
}

int32_t gdr_abi_version(void) { return GDR_ABI_VERSION; }

}  // extern "C"
