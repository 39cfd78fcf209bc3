/*
 * gdr.h -- the C ABI of libgdr, a B200 (sm_100a) implementation of bunsen's
 * gated delta rule.
 *
 * Each entry point replaces one method of bunsen's Rust operator
 * `GatedDeltaRule` (crates/public/bunsen/src/ops/transformers/
 * linear_attention/delta_rule.rs):
 *
 *   gdr_recurrent  <- GatedDeltaRule::recurrent   (delta_rule.rs:182-209)
 *   gdr_chunked    <- GatedDeltaRule::chunked     (delta_rule.rs:223-310)
 *   gdr_mixed      <- no single counterpart: one launch that runs what
 *                     GatedDeltaNet::forward (blocks/transformers/mixers/
 *                     gated_delta_net.rs:428-433) dispatches per call --
 *                     `chunked` for prefill segments and `recurrent` for
 *                     single-token decode rows -- for many sequences at once.
 *
 * The argument order is the Rust operator's: q, k, v, g, beta, state; the
 * rule's options (`qk_l2norm_eps`, `chunk_size`, delta_rule.rs:52-60) travel
 * in `gdr_params`, as `&self` does in Rust. Results: the output and the state
 * after the last position.
 *
 * Conventions
 *  - Every pointer is a device pointer (CUDA global memory), except `params`
 *    (and the other parameter structs), which live on the host, and the
 *    buffers of gdr_chunked_host. Nothing here allocates device memory
 *    except where an entry point says so.
 *  - `stream` is a `cudaStream_t` passed as `void*` (NULL: the legacy default
 *    stream). Every call is asynchronous on it; a returned GDR_OK means the
 *    work was enqueued, not that it finished.
 *  - Layouts are bunsen's logical layouts, row-major and contiguous:
 *      q, k        [B, T, H_qk, d_k]   (dense)   or [T_total, H_qk, d_k] (packed)
 *      v, out      [B, T, H_v,  d_v]             or [T_total, H_v,  d_v]
 *      g, beta     [B, T, H_v]  f32              or [T_total, H_v]
 *      state_in,
 *      state_out   [B, H_v, d_k, d_v] f32        or [n_seqs, H_v, d_k, d_v]
 *    A dense batch has cu_seqlens == NULL; a packed ragged batch passes
 *    `cu_seqlens` (device int32, n_seqs + 1 non-decreasing offsets from 0 to
 *    T_total).
 *  - Heads: bunsen's rule sees q and k already repeated to H_v heads
 *    (`repeat_interleave`, ops/repeat.rs:51-66, applied at
 *    gated_delta_net.rs:404-419). Here q and k keep their H_qk heads and value
 *    head h reads key head h / (H_v / H_qk), which is the same arithmetic
 *    without the copy; H_qk == H_v is bunsen's signature exactly.
 *  - dtypes: q, k, v share `params->dtype`; `out` is written in that dtype
 *    (bunsen narrows the output to q's dtype, delta_rule.rs:207, 304). g,
 *    beta and the states are f32, the dtype the rule runs in
 *    (burner/tensor/widening.rs:60); f64 in the f64 entry points.
 *  - `state_in` may be NULL (zeros, delta_rule.rs:330). `state_out` may equal
 *    `state_in` (an in-place update); bunsen itself never writes into a state
 *    (linear_attention/state.rs:201-204), so a caller that shares states must
 *    pass a fresh `state_out`.
 *  - Errors never cross the ABI as exceptions. Bunsen panics on a shape
 *    mismatch (delta_rule.rs:135-150) or a zero chunk size (:233); here those
 *    return GDR_ERR_INVALID and launch nothing.
 */
#ifndef GDR_H
#define GDR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDR_ABI_VERSION 3

typedef enum gdr_status {
    GDR_OK = 0,
    GDR_ERR_INVALID = 1,     /* bad shape, pointer or option (bunsen: panic) */
    GDR_ERR_UNSUPPORTED = 2, /* valid, but no kernel for these dims/dtypes   */
    GDR_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed         */
    GDR_ERR_TIMEOUT = 4,     /* a bounded device-side wait ran out           */
    GDR_ERR_CAPACITY = 5     /* more than a fixed-size entry point can take  */
} gdr_status;

/* q, k, v and out share one dtype. bunsen widens half-precision inputs to f32
 * (burner/tensor/widening.rs:58-60) and narrows the output back: bf16 runs
 * take bf16 operands on the tensor cores with f32 accumulation; f16 runs
 * compute in f32 on the CUDA-core kernels, as f32 runs do. f64, which bunsen
 * keeps as its compute dtype (g, beta and the state included), has its own
 * entry points, gdr_recurrent_f64 and gdr_chunked_f64. */
typedef enum gdr_dtype {
    GDR_DTYPE_F32 = 0,
    GDR_DTYPE_BF16 = 1,
    GDR_DTYPE_F16 = 2,
    GDR_DTYPE_F64 = 3  /* gdr_recurrent_f64 / gdr_chunked_f64 only */
} gdr_dtype;

/* Which kernel family runs a chunked call. AUTO picks the tensor-core kernels
 * for bf16, d_k = d_v = 128, chunk 64 -- split into segments when some
 * sequence could be longer than twice the smallest segment worth running
 * (see GDR_ALGO_TENSOR_SPLIT) -- and the CUDA-core f32 kernel otherwise.
 * Shapes that kernel does not take (chunk above 64, or d_k or d_v above 128,
 * up to 256) run on the recurrent kernel, under AUTO and CUDA_CORE alike:
 * bunsen's chunked and recurrent forms are the same rule and agree to f32
 * rounding (delta_rule.rs:549-608), the chunk size only changing how. */
typedef enum gdr_algo {
    GDR_ALGO_AUTO = 0,
    GDR_ALGO_CUDA_CORE = 1,   /* f32 FFMA throughout: f32 and f16 runs, any dims
                                 up to 256                                    */
    GDR_ALGO_TENSOR = 2,      /* tcgen05/TMEM, bf16 operands, f32 accumulate;
                                 one pass per (sequence, head)                 */
    GDR_ALGO_TENSOR_SPLIT = 3 /* the same kernel over segments of the long
                                 sequences, chained by their state transitions
                                 (sequence-parallel); allocates a stream-ordered
                                 scratch from a library-owned pool             */
} gdr_algo;

typedef struct gdr_params {
    int32_t batch;      /* B of a dense batch; ignored when cu_seqlens != NULL */
    int32_t seq_len;    /* T of a dense batch, or T_total of a packed one      */
    int32_t n_seqs;     /* sequences of a packed batch (cu_seqlens has +1)     */
    int32_t heads_qk;   /* H_qk: key/query heads                               */
    int32_t heads_v;    /* H_v: value heads, the rule's H; H_qk divides it     */
    int32_t d_k;        /* key width per head                                  */
    int32_t d_v;        /* value width per head                                */
    int32_t chunk_size; /* GatedDeltaRule::chunk_size (bunsen default 64)      */
    int32_t use_l2norm; /* qk_l2norm_eps is Some(l2norm_eps)                   */
    double l2norm_eps;  /* bunsen default 1e-6                                 */
    int32_t dtype;      /* gdr_dtype of q, k, v and out                        */
    int32_t algo;       /* gdr_algo, chunked calls only                        */
    int32_t split_chunks; /* GDR_ALGO_TENSOR_SPLIT / AUTO: segment length in
                             chunks; 0 lets the call choose from the lengths  */
} gdr_params;

/* The rule one position at a time (GatedDeltaRule::recurrent,
 * delta_rule.rs:182-209). A decode step is a call with T = 1 (dense) or with
 * every sequence of length 1 (packed). */
gdr_status gdr_recurrent(const gdr_params* params, const void* q, const void* k, const void* v,
                         const float* g, const float* beta, const float* state_in, void* out,
                         float* state_out, const int32_t* cu_seqlens, void* stream);

/* The rule a chunk at a time (GatedDeltaRule::chunked, delta_rule.rs:223-310).
 * A sequence's last chunk may be short. Agrees with gdr_recurrent. */
gdr_status gdr_chunked(const gdr_params* params, const void* q, const void* k, const void* v,
                       const float* g, const float* beta, const float* state_in, void* out,
                       float* state_out, const int32_t* cu_seqlens, void* stream);

/* The two forms for f64 inputs (params->dtype = GDR_DTYPE_F64): q, k, v, g,
 * beta, out and both states in f64, every product in f64 on the CUDA cores,
 * as bunsen computes when its inputs are f64 (widening.rs:58-60 keeps f64).
 * Both run the recurrent kernel: the chunked form is the same rule, equal to
 * the recurrent one up to rounding (delta_rule.rs:549-608), so the chunk size
 * is checked (> 0) but changes nothing. Any d_k, d_v up to 256. */
gdr_status gdr_recurrent_f64(const gdr_params* params, const double* q, const double* k,
                             const double* v, const double* g, const double* beta,
                             const double* state_in, double* out, double* state_out,
                             const int32_t* cu_seqlens, void* stream);
gdr_status gdr_chunked_f64(const gdr_params* params, const double* q, const double* k,
                           const double* v, const double* g, const double* beta,
                           const double* state_in, double* out, double* state_out,
                           const int32_t* cu_seqlens, void* stream);

/* gdr_chunked on HOST buffers: every pointer (cu_seqlens included) is host
 * memory, pinned for the copies to overlap. The call copies groups of whole
 * sequences in, runs them and copies their outputs and final states out,
 * three groups in flight on library-owned streams, so copies in, kernels and
 * copies out overlap; device scratch comes from the library's pool. Work is
 * ordered after earlier work on `stream` and later work on `stream` waits for
 * it; the host buffers must stay valid (and `out` / `state_out` unread) until
 * `stream` has passed the call. A packed batch's cu_seqlens must start at 0,
 * not decrease and end at seq_len (T_total). No counterpart in the reference:
 * it serves callers whose tensors live in host memory. */
gdr_status gdr_chunked_host(const gdr_params* params, const void* q, const void* k, const void* v,
                            const float* g, const float* beta, const float* state_in, void* out,
                            float* state_out, const int32_t* cu_seqlens, void* stream);

/* ---- The layer's steps around the rule ------------------------------------
 * GatedDeltaNet::forward (blocks/transformers/mixers/gated_delta_net.rs:396-440)
 * runs, around the rule: a causal depthwise convolution of in_proj_qkv(x) with
 * silu, split into q, k, v; the gates from in_proj_a(x), in_proj_b(x); and a
 * gated RMS norm of the rule's output with in_proj_z(x). */

/* The short convolution (causal_depthwise_conv1d, ops/transformers/
 * linear_attention/causal_conv.rs:36-69): y[t, c] = sum_j w[c, j] x[t - (K-1) + j, c],
 * the K - 1 inputs before a sequence's first position taken from its state
 * (zeros when state_in is NULL). x is dense [B, T, C] or packed [T_total, C]
 * (cu_seqlens); weight [C, K], oldest tap first; states [N, K - 1, C] f32,
 * oldest first (DeltaNetState.conv, state.rs:88). Channels [0, split0) are
 * written to out0 as [.., split0], [split0, split1) to out1, the rest to out2
 * (the layer's q / k / v split; split0 = split1 = C writes one [.., C]
 * output). `silu` applies the layer's activation. state_out (NULL: none) gets
 * the last K - 1 inputs of [state, x] and may equal state_in. Any shape runs;
 * bf16 or f16 with C, split0 and split1 multiples of 8, x and the outputs 16-byte
 * aligned and the states 8-byte aligned takes the fast kernel (eight channels
 * per thread, 16-byte accesses), the layer's own shapes among them. */
typedef struct gdr_conv_params {
    int32_t batch;    /* B of a dense batch; ignored when cu_seqlens != NULL */
    int32_t seq_len;  /* T of a dense batch, or T_total of a packed one */
    int32_t n_seqs;   /* sequences of a packed batch */
    int32_t channels; /* C */
    int32_t taps;     /* K, 2 to 8 */
    int32_t split0, split1;
    int32_t silu;
    int32_t dtype;    /* gdr_dtype of x, weight and the outputs */
} gdr_conv_params;

gdr_status gdr_causal_conv1d(const gdr_conv_params* params, const void* x, const void* weight,
                             const float* state_in, void* out0, void* out1, void* out2,
                             float* state_out, const int32_t* cu_seqlens, void* stream);

/* Optional inputs of a rule call that also runs the layer's gates and gated
 * norm. gate_a != NULL: the call's g and beta must be NULL and are computed
 * per position and value head as g = -exp(a_log[h]) softplus(a + dt_bias[h]),
 * beta = sigmoid(b) (gated_delta_net.rs:422-426), from a, b [T, H_v] in
 * gate_dtype and a_log, dt_bias [H_v] f32. norm_z != NULL: `out` receives
 * rmsnorm(core) * norm_weight * silu(z) over each head's d_v features
 * (gated_delta_net.rs:439-440, GatedNorm), core being the rule's output in q's
 * dtype, z [T, H_v, d_v] in q's dtype, norm_weight [d_v] f32. */
typedef struct gdr_layer_io {
    const void* gate_a;
    const void* gate_b;
    const float* a_log;
    const float* dt_bias;
    int32_t gate_dtype;
    const void* norm_z;
    const float* norm_weight;
    double norm_eps;
} gdr_layer_io;

/* gdr_chunked / gdr_recurrent with the layer's gates and gated norm (io may
 * be NULL: the plain call). */
gdr_status gdr_chunked_layer(const gdr_params* params, const void* q, const void* k,
                             const void* v, const float* g, const float* beta,
                             const gdr_layer_io* io, const float* state_in, void* out,
                             float* state_out, const int32_t* cu_seqlens, void* stream);
gdr_status gdr_recurrent_layer(const gdr_params* params, const void* q, const void* k,
                               const void* v, const float* g, const float* beta,
                               const gdr_layer_io* io, const float* state_in, void* out,
                               float* state_out, const int32_t* cu_seqlens, void* stream);

/* The layer's gated RMS norm on its own (gated_delta_net.rs:439-440, GatedNorm):
 * out = rmsnorm(x) * weight * silu(z) over each row of `width` features; x, z
 * and out [rows, width] in `dtype`, weight [width] f32; out may be x. */
gdr_status gdr_gated_norm(int64_t rows, int32_t width, const void* x, const void* z,
                          const float* weight, double eps, int32_t dtype, void* out,
                          void* stream);

/* gdr_mixed with the layer's gates and gated norm, fused into its prefill
 * segments and decode rows (io as for gdr_chunked_layer; NULL: gdr_mixed). */
gdr_status gdr_mixed_layer(const gdr_params* params, const void* q, const void* k,
                           const void* v, const float* g, const float* beta,
                           const gdr_layer_io* io, float* state_pool,
                           const int32_t* state_slots, int32_t n_slots, void* out,
                           const int32_t* cu_seqlens, void* workspace, size_t workspace_bytes,
                           void* stream);

/* DeltaNetState::reorder (state.rs:112-135) on device: row r of dst becomes row
 * sources[r] of src, for `rows` rows of row_bytes bytes (a multiple of 4);
 * sources is device memory; src and dst must not overlap. A source outside
 * [0, src_rows) leaves its row untouched and is reported by gdr_device_error
 * as GDR_ERR_INVALID. Snapshots (state.rs:201-240) are plain copies of the
 * state buffers. */
gdr_status gdr_state_reorder(const void* src, void* dst, const int32_t* sources, int32_t rows,
                             int32_t src_rows, size_t row_bytes, void* stream);

/* How many kernels a gdr_chunked call with these parameters launches (0 when
 * there is nothing to run; 4 for the split form: plan, two passes, scan), or
 * -1 when the call would be rejected. `packed`: the call passes cu_seqlens.
 * No counterpart in the reference; it lets a caller count device launches. */
int32_t gdr_chunked_launches(const gdr_params* params, int32_t packed);

/* A continuous batch in one launch: the packed batch of `cu_seqlens`, whose
 * sequences of length 1 are decode rows (run as gdr_recurrent would) and whose
 * longer sequences are prefill segments (run as gdr_chunked would); sequences
 * of length 0 are left alone. Sequence s reads and writes its state in place
 * at `state_pool[state_slots[s]]` ([n_slots, H_v, d_k, d_v] f32);
 * `state_slots` NULL means slot s. A slot holds its sequence's state on entry
 * (a fresh sequence's slot holds zeros); two sequences of one call must not
 * share a slot. A slot outside [0, n_slots) skips its sequence and is
 * reported by gdr_device_error as GDR_ERR_INVALID.
 * Work runs from a device-side work list -- prefill segments first, longest
 * first, then decode rows -- that the call builds in `workspace`: device
 * memory of at least gdr_mixed_workspace_size(params) bytes, 4-byte aligned,
 * owned by the caller; calls that overlap on the GPU need separate
 * workspaces. Kernel family: bf16, d_k = d_v = 128, chunk 64
 * (GDR_ERR_UNSUPPORTED otherwise); `out` as for gdr_chunked. */
size_t gdr_mixed_workspace_size(const gdr_params* params);
gdr_status gdr_mixed(const gdr_params* params, const void* q, const void* k, const void* v,
                     const float* g, const float* beta, float* state_pool,
                     const int32_t* state_slots, int32_t n_slots, void* out,
                     const int32_t* cu_seqlens, void* workspace, size_t workspace_bytes,
                     void* stream);

/* gdr_mixed for callers that cannot allocate device memory. No counterpart in
 * the reference: bunsen allocates through burn on every call.
 *
 * Some callers may not allocate at all: a serving loop whose device memory
 * is budgeted up front, code running under another framework's memory pool,
 * or a host thread that must not take the allocator's locks or the device
 * synchronisation a cudaMalloc/cudaFree can imply. This entry point takes the
 * same arguments as gdr_mixed minus the workspace and allocates nothing: its
 * work list lives in a fixed array inside the library, sized for at most
 * GDR_MIXED_NOALLOC_MAX_SEQS sequences (64 KiB of device memory that every GPU
 * loading the library holds until the process exits). A call with more
 * sequences returns GDR_ERR_CAPACITY and launches nothing.
 *
 * The first call on each device looks the array's device address up
 * (cudaGetSymbolAddress); make that first call before any stream capture on
 * that device. All calls on a device share the array: two calls whose work
 * can overlap on the GPU (different streams with no ordering between them)
 * race on it and must not be issued. */
#define GDR_MIXED_NOALLOC_MAX_SEQS 16384
gdr_status gdr_mixed_noalloc(const gdr_params* params, const void* q, const void* k,
                             const void* v, const float* g, const float* beta, float* state_pool,
                             const int32_t* state_slots, int32_t n_slots, void* out,
                             const int32_t* cu_seqlens, void* stream);

/* What the kernels of this library recorded on the device since the last
 * call (the record is then cleared): GDR_ERR_TIMEOUT if one gave up a bounded
 * wait, else GDR_ERR_INVALID if gdr_mixed met a state slot outside its pool,
 * else GDR_OK. Synchronous: waits for the device's outstanding work. */
gdr_status gdr_device_error(void);

/* A self-test of failure detection: launches one thread that waits, at most
 * `limit_ns` (0 < limit_ns <= 1e8, else GDR_ERR_INVALID), for a device-side
 * barrier nothing completes, through the same bounded wait the kernels use.
 * The wait gives up, the kernel returns, and the next gdr_device_error()
 * reports GDR_ERR_TIMEOUT; the context stays usable. */
gdr_status gdr_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Scratch memory. Split calls (GDR_ALGO_TENSOR_SPLIT, and AUTO when it
 * splits), gdr_chunked_host and the layer calls whose gates are not fused
 * take their device scratch from a stream-ordered pool the library owns, one
 * per device. Freed scratch stays reserved in that pool so that the next call
 * reuses it: up to about 2 GiB of segment states for split calls, three groups'
 * worth of buffers for gdr_chunked_host. gdr_release_scratch returns the
 * current device's unused pool memory to the driver: it waits for the
 * device's outstanding work, then trims the pool (GDR_OK when the device has
 * no pool). The next call that needs scratch reserves it again.
 *
 * The library keeps per-device handles for the life of the process (the pool,
 * gdr_chunked_host's worker streams, gdr_mixed_noalloc's array address), so a
 * cudaDeviceReset after the first call on a device is not supported. */
gdr_status gdr_release_scratch(void);

/* A short English description of a status. */
const char* gdr_status_string(gdr_status status);

/* GDR_ABI_VERSION of the loaded library. */
int32_t gdr_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDR_H */
