// The extern "C" entry points of include/gdr.h: argument checks (bunsen's
// shape contracts, delta_rule.rs:135-150 and :233, become GDR_ERR_INVALID),
// then the kernel that serves the call.
#include <cmath>

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
cudaError_t take_device_error(int* flag);
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

// Checks what the host can check and fills the kernels' descriptor.
gdr_status make_problem(const gdr_params* params, const int32_t* cu_seqlens, Problem& p) {
    if (params == nullptr) return GDR_ERR_INVALID;
    const gdr_params& a = *params;
    if (a.heads_qk <= 0 || a.heads_v <= 0 || a.heads_v % a.heads_qk != 0) return GDR_ERR_INVALID;
    if (a.d_k <= 0 || a.d_v <= 0 || a.seq_len < 0) return GDR_ERR_INVALID;
    if (a.dtype != GDR_DTYPE_F32 && a.dtype != GDR_DTYPE_BF16) return GDR_ERR_INVALID;
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
bool io_ok(const Problem& p, const void* q, const void* k, const void* v, const float* g,
           const float* beta, const void* out, const float* state_out) {
    const bool tokens = total_tokens(p) > 0;
    return (!tokens || (q && k && v && g && beta && out)) && (p.n_seqs == 0 || state_out);
}

gdr_status from_cuda(cudaError_t e) { return e == cudaSuccess ? GDR_OK : GDR_ERR_CUDA; }

enum class ChunkedPath { kNothing, kPassThrough, kTensor, kSplit, kCudaCore };

// Which kernels a gdr_chunked call runs: the checks of everything but the
// buffers, then the algorithm (GDR_ALGO_AUTO: the tensor-core kernels where
// they apply -- split into segments when that may help -- else the f32 one).
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
    if (algo == GDR_ALGO_TENSOR || algo == GDR_ALGO_TENSOR_SPLIT) {
        if (!tc_ok) return GDR_ERR_UNSUPPORTED;
        path = algo == GDR_ALGO_TENSOR ? ChunkedPath::kTensor : ChunkedPath::kSplit;
    } else if (algo == GDR_ALGO_CUDA_CORE) {
        if (!ffma_ok) return GDR_ERR_UNSUPPORTED;
        path = ChunkedPath::kCudaCore;
    } else {
        if (!tc_ok && !ffma_ok) return GDR_ERR_UNSUPPORTED;
        path = !tc_ok ? ChunkedPath::kCudaCore
               : (params->split_chunks > 0 || gdr::split_may_help(p)) ? ChunkedPath::kSplit
                                                                       : ChunkedPath::kTensor;
    }
    if (p.n_seqs == 0) path = ChunkedPath::kNothing;
    else if (total_tokens(p) == 0) path = ChunkedPath::kPassThrough;
    return GDR_OK;
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
    if (p.d_k > 256 || p.d_v > 256) return GDR_ERR_UNSUPPORTED;
    if (p.n_seqs == 0) return GDR_OK;
    return from_cuda(gdr::launch_recurrent(p, params->dtype, q, k, v, g, beta, state_in, out,
                                           state_out, static_cast<cudaStream_t>(stream)));
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
    int flag = 0;
    if (gdr::take_device_error(&flag) != cudaSuccess) return GDR_ERR_CUDA;
    if (flag & 1) return GDR_ERR_TIMEOUT;
    return (flag & 2) ? GDR_ERR_INVALID : GDR_OK;
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
