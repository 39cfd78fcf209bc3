// GatedDeltaRule::chunked (delta_rule.rs:223-310) on the sm_100a tensor cores.
//
// bf16 q/k/v, d_k = d_v = 128, chunk C = 64; f32 g, beta, state, f32
// accumulation everywhere. One CTA (128 threads, one TMEM lane each) per
// (sequence, value head) walks the sequence's chunks in order; the state
// lives in TMEM for the whole sequence and touches HBM once on each end.
//
// Every contraction of a chunk is one tcgen05.mma group with M = 128 (the
// feature axis, or the 64 keys stacked on the 64 queries), so the tensor
// core always runs full-height tiles. The state is kept transposed,
// S^T [d_v, d_k], so that it is the accumulator of its own update:
//
//   G1  [K;Q] K^T            -> TMEM R0 [128 x 64]   Gram of keys / queries
//        (CUDA cores: norms, decay mask, L = strict_lower(.), intra,
//         A = (I + L)^-1 by a blocked forward substitution)
//   G2  V^T (A diag(beta))^T                -> R1  U^T       [d_v x C]
//       K^T (A diag(beta e^gamma / |k|))^T  -> R0  W^T       [d_k x C]
//        (CUDA cores: S^T -> bf16 operand, S^T <- e^gamma_C S^T; W^T -> bf16)
//   G3  R1 += -(S^T W^T)        V_new^T = U^T - (W S)^T
//       S^T Q^T                 -> R0  (Q S)^T
//        (CUDA cores: V_new^T -> bf16, and a copy scaled by e^(gamma_C -
//         gamma_t) / |k_t| per position)
//   G4  V_new^T intra^T         -> R1  (intra V_new)^T
//   G5  S^T += (V_new^T o r) K  the state update
//        (CUDA cores: O^T = (Q S)^T diag(e^gamma / |q| sqrt(d_k)) + R1)
//
// q and k enter the tensor core raw; their L2 norms (delta_rule.rs:112-123)
// and the 1/sqrt(d_k) scale are applied as per-position factors on the
// CUDA-core side, so no pass rewrites the input tiles. Positions past a
// sequence's end take beta = g = 0, which makes them write nothing
// (delta_rule.rs:241-262), whatever the tile holds there.
//
// Operand tiles are 128-byte swizzled; TMA writes the input tiles, the
// CUDA-core stages write the rest with the same swizzle. Shared memory:
//   KQ  32 KiB  [k-block][K rows 0-63 | Q rows 64-127] x 128 B  (TMA)
//   VB  16 KiB  V (TMA) -> W^T operand -> output staging
//   AB  16 KiB  A diag(beta) | A diag(beta e^gamma/|k|) -> intra operand
//   ST  32 KiB  solve scratch (f32) -> S^T operand -> V_new^T operands
// ~98 KiB, so two CTAs share an SM (and its 512 TMEM columns).
#include <cudaTypedefs.h>

#include "gdr_common.cuh"
#include "gdr_sm100.cuh"

namespace gdr {

__device__ int g_tc_error;  // set when a bounded wait in the kernel ran out

namespace {

using namespace sm100;

constexpr int kC = 64;       // chunk
constexpr int kD = 128;      // d_k = d_v
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColR0 = 128, kColR1 = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

constexpr uint32_t kOffKQ = 0, kOffVB = 32768, kOffAB = 49152, kOffST = 65536;
constexpr uint32_t kOffMisc = 98304;
constexpr uint32_t kTileBytes = 8192;  // one 64 x 64 bf16 TMA box
constexpr uint32_t kSmemBytes = kOffMisc + 2048 + 1024;  // + alignment slack

struct Misc {
    float gam[kC];   // cumulative log decay within the chunk
    float bet[kC];   // beta (0 past the end)
    float fk[kC];    // 1 / |k_t|
    float fq[kC];    // 1 / (|q_t| sqrt(d_k))
    float wk[kC];    // beta_t e^gamma_t / |k_t|
    float rr[kC];    // e^(gamma_C - gamma_t) / |k_t|
    float cq[kC];    // e^gamma_t / (|q_t| sqrt(d_k))
    uint64_t bar_tma, bar_mma;
    uint32_t tmem_base;
    int failed;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&x);
}

// Writes 64 f32 values as one 128-byte swizzled row (8 chunks of 8 bf16).
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int row, const float* x) {
    uint8_t* base = tile + row * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = pack_bf16(x[8 * c + 0], x[8 * c + 1]);
        v.y = pack_bf16(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_bf16(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_bf16(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(base + ((c ^ (row & 7)) << 4)) = v;
    }
}

// Sum of squares of a 128-element bf16 row stored as two 128-B swizzled
// halves (the swizzle only permutes 16-B chunks within a row).
__device__ __forceinline__ float row_sumsq(const uint8_t* half0, const uint8_t* half1) {
    float acc = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4* p = reinterpret_cast<const uint4*>(h ? half1 : half0);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 u = p[c];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
                acc = fmaf(f.x, f.x, acc);
                acc = fmaf(f.y, f.y, acc);
            }
        }
    }
    return acc;
}

// A = (I + L)^-1 for the strictly lower 64 x 64 L in `Lf` (f32, row-major),
// into `X` (f32, row-major, zero above the diagonal). 16 x 16 diagonal
// blocks by forward substitution, then the off-diagonal blocks level by
// level: X_ij = -X_ii sum_{k=j}^{i-1} L_ik X_kj. `Tm` holds 3 16 x 16 f32
// blocks of scratch.
__device__ void unit_lower_inverse_64(const float* Lf, float* X, float* Tm, int tid) {
    if (tid < 64) {
        const int b = tid >> 4, m = tid & 15;
        const float* Lb = Lf + (16 * b) * kC + 16 * b;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float acc = (r == m) ? 1.f : 0.f;
#pragma unroll
            for (int j = 0; j < r; ++j) acc = fmaf(-Lb[r * kC + j], x[j], acc);
            x[r] = acc;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) X[(16 * b + r) * kC + 16 * b + m] = x[r];
    } else {
        // Zero every block above the block diagonal.
        for (int e = tid - 64; e < kC * kC; e += 64) {
            const int i = e / kC, j = e % kC;
            if ((j >> 4) > (i >> 4)) X[e] = 0.f;
        }
    }
    __syncthreads();
    // Levels 1..3: blocks (j + lvl, j).
#pragma unroll 1
    for (int lvl = 1; lvl < 4; ++lvl) {
        const int nblk = 4 - lvl;
        for (int e = tid; e < nblk * 256; e += kThreads) {
            const int jb = e >> 8, r = (e >> 4) & 15, c = e & 15;
            const int ib = jb + lvl;
            float acc = 0.f;
            for (int kb = jb; kb < ib; ++kb) {
                const float* Lrow = Lf + (16 * ib + r) * kC + 16 * kb;
                const float* Xcol = X + (16 * kb) * kC + 16 * jb + c;
#pragma unroll
                for (int k = 0; k < 16; ++k) acc = fmaf(Lrow[k], Xcol[k * kC], acc);
            }
            Tm[e] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nblk * 256; e += kThreads) {
            const int jb = e >> 8, r = (e >> 4) & 15, c = e & 15;
            const int ib = jb + lvl;
            const float* Xrow = X + (16 * ib + r) * kC + 16 * ib;
            const float* T = Tm + (jb << 8) + c;
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) acc = fmaf(Xrow[k], T[k * 16], acc);
            X[(16 * ib + r) * kC + 16 * jb + c] = -acc;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads, 2)
chunked_tc(const Problem p, const __grid_constant__ CUtensorMap tm_q,
           const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
           const float* __restrict__ g, const float* __restrict__ beta, const float* state_in,
           __nv_bfloat16* __restrict__ out, float* state_out) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* KQ = smem + kOffKQ;
    uint8_t* VB = smem + kOffVB;
    uint8_t* AB = smem + kOffAB;
    uint8_t* ST = smem + kOffST;
    Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, s = blockIdx.y;
    const int hq = h / p.group;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t len = t1 - t0;
    const int n_chunks = static_cast<int>((len + kC - 1) / kC);

    if (tid == 0) {
        mbar_init(&ms.bar_tma, 1);
        mbar_init(&ms.bar_mma, 1);
        ms.failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ms.tmem_base;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    const uint32_t tS = lane_addr + kColS, tR0 = lane_addr + kColR0, tR1 = lane_addr + kColR1;

    // The initial state, transposed into TMEM: lane d holds S[:, d].
    const int64_t head_state = (static_cast<int64_t>(s) * p.heads_v + h) * kD * kD;
    {
        const int d = tid;
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
            float x[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
                x[i] = state_in ? state_in[head_state + (cb * 32 + i) * kD + d] : 0.f;
            tmem_st32(tS + cb * 32, x);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();

    uint32_t ph_tma = 0, ph_mma = 0;
    bool ok = true;
    const uint32_t sKQ = smem_u32(KQ), sVB = smem_u32(VB), sAB = smem_u32(AB), sST = smem_u32(ST);

    // Waits on an mbarrier phase; on time-out records it and stops the walk.
    auto wait = [&](uint64_t* bar, uint32_t& ph) {
        if (!mbar_wait(bar, ph, kWaitLimitNs)) {
            ms.failed = 1;
            atomicExch(&g_tc_error, 1);
        }
        ph ^= 1u;
    };

#pragma unroll 1
    for (int ci = 0; ci < n_chunks && ok; ++ci) {
        const int64_t tok0 = t0 + static_cast<int64_t>(ci) * kC;
        const int valid = static_cast<int>(len - static_cast<int64_t>(ci) * kC < kC
                                               ? len - static_cast<int64_t>(ci) * kC
                                               : kC);
        // (1) The chunk's tiles: K and Q stacked per 64-wide k-block, then V.
        if (tid == 0) {
            fence_proxy_async();
            mbar_expect_tx(&ms.bar_tma, 6 * kTileBytes);
            const int tok = static_cast<int>(tok0);
            tma_load_3d(KQ + 0 * kTileBytes, &tm_k, &ms.bar_tma, 0, hq, tok);
            tma_load_3d(KQ + 1 * kTileBytes, &tm_q, &ms.bar_tma, 0, hq, tok);
            tma_load_3d(KQ + 2 * kTileBytes, &tm_k, &ms.bar_tma, 64, hq, tok);
            tma_load_3d(KQ + 3 * kTileBytes, &tm_q, &ms.bar_tma, 64, hq, tok);
            tma_load_3d(VB + 0 * kTileBytes, &tm_v, &ms.bar_tma, 0, h, tok);
            tma_load_3d(VB + 1 * kTileBytes, &tm_v, &ms.bar_tma, 64, h, tok);
            if (ci + 1 < n_chunks) {
                const int nt = tok + kC;
                tma_prefetch_3d(&tm_k, 0, hq, nt);
                tma_prefetch_3d(&tm_k, 64, hq, nt);
                tma_prefetch_3d(&tm_q, 0, hq, nt);
                tma_prefetch_3d(&tm_q, 64, hq, nt);
                tma_prefetch_3d(&tm_v, 0, h, nt);
                tma_prefetch_3d(&tm_v, 64, h, nt);
            }
        }
        // (2) Gates, zero past the end; the cumulative decay by a warp scan.
        if (tid < kC) {
            const bool in = tid < valid;
            const int64_t gi = (tok0 + tid) * p.heads_v + h;
            ms.gam[tid] = in ? g[gi] : 0.f;
            ms.bet[tid] = in ? beta[gi] : 0.f;
        }
        __syncthreads();
        if (warp == 0) {
            const float a = ms.gam[2 * lane], b = ms.gam[2 * lane + 1];
            float incl = a + b;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const float excl = incl - (a + b);
            ms.gam[2 * lane] = excl + a;
            ms.gam[2 * lane + 1] = excl + a + b;
        }
        wait(&ms.bar_tma, ph_tma);
        // (3) Query norms from the raw Q rows (threads 64..127, row tid-64).
        if (tid >= kC) {
            const int i = tid - kC;
            const float ss = row_sumsq(KQ + 1 * kTileBytes + i * 128, KQ + 3 * kTileBytes + i * 128);
            ms.fq[i] = l2_factor(p, ss) * p.q_scale;
        }
        // (4) G1: [K;Q] K^T -> R0.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id = idesc_bf16(128, 64, 0, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
                umma_bf16(tbase + kColR0, sdesc_sw128(sKQ + off, 16, 1024),
                          sdesc_sw128(sKQ + off, 16, 1024), id, ks > 0);
            }
            umma_commit(&ms.bar_mma);
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (5) Gram rows: lanes 0-63 k_i . k_j, lanes 64-127 q_i . k_j.
        float row[kC];
        {
            float a[32], b[32];
            tmem_ld32(tR0, a);
            tmem_ld32(tR0 + 32, b);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                row[j] = a[j];
                row[32 + j] = b[j];
            }
        }
        if (tid < kC) {
            float diag = 0.f;
#pragma unroll
            for (int j = 0; j < kC; ++j)
                if (j == tid) diag = row[j];
            ms.fk[tid] = l2_factor(p, diag);
        }
        __syncthreads();
        float* Lf = reinterpret_cast<float*>(ST);
        float* X = reinterpret_cast<float*>(ST + 16384);
        float* Tm = reinterpret_cast<float*>(AB);
        if (tid < kC) {
            const int i = tid;
            const float gi = ms.gam[i], ci_ = ms.bet[i] * ms.fk[i];
            float* Lrow = Lf + i * kC;
#pragma unroll
            for (int j = 0; j < kC; ++j)
                Lrow[j] = (j < i) ? ci_ * ms.fk[j] * row[j] * __expf(gi - ms.gam[j]) : 0.f;
            const float last = ms.gam[kC - 1];
            ms.wk[i] = ms.bet[i] * __expf(gi) * ms.fk[i];
            ms.rr[i] = __expf(last - gi) * ms.fk[i];
        } else {
            const int i = tid - kC;
            const float gi = ms.gam[i], fqi = ms.fq[i];
#pragma unroll
            for (int j = 0; j < kC; ++j)
                row[j] = (j <= i) ? fqi * ms.fk[j] * row[j] * __expf(gi - ms.gam[j]) : 0.f;
            ms.cq[i] = __expf(gi) * fqi;
        }
        __syncthreads();
        // (6) A = (I + L)^-1.
        unit_lower_inverse_64(Lf, X, Tm, tid);
        // (7) The two column scalings of A, as bf16 K-major B operands.
        {
            const int i = tid & 63;
            const float* Xrow = X + i * kC;
            float a[kC];
            if (tid < kC) {
#pragma unroll
                for (int j = 0; j < kC; ++j) a[j] = Xrow[j] * ms.bet[j];
            } else {
#pragma unroll
                for (int j = 0; j < kC; ++j) a[j] = Xrow[j] * ms.wk[j];
            }
            store_row_sw128(AB + (tid < kC ? 0 : kTileBytes), i, a);
        }
        fence_proxy_async();
        __syncthreads();
        // (8) G2: U^T = V^T Au^T -> R1; W^T = K^T Aw^T -> R0.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id = idesc_bf16(128, 64, 1, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tbase + kColR1, sdesc_sw128(sVB + ks * 2048, 8192, 1024),
                          sdesc_sw128(sAB + ks * 32, 16, 1024), id, ks > 0);
            }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tbase + kColR0, sdesc_sw128(sKQ + ks * 2048, 16384, 1024),
                          sdesc_sw128(sAB + kTileBytes + ks * 32, 16, 1024), id, ks > 0);
            }
            umma_commit(&ms.bar_mma);
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (9) S^T -> bf16 operand (ST), S^T <- e^gamma_C S^T; W^T -> bf16 (VB);
        //     intra rows -> bf16 (AB, over the consumed A diag(beta)).
        {
            const int d = tid;
            const float decay = __expf(ms.gam[kC - 1]);
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                float x[64];
                float a[32], b[32];
                tmem_ld32(tS + half * 64, a);
                tmem_ld32(tS + half * 64 + 32, b);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    x[i] = a[i];
                    x[32 + i] = b[i];
                }
                store_row_sw128(ST + half * 16384, d, x);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    a[i] *= decay;
                    b[i] *= decay;
                }
                tmem_st32(tS + half * 64, a);
                tmem_st32(tS + half * 64 + 32, b);
            }
            float w[64];
            {
                float a[32], b[32];
                tmem_ld32(tR0, a);
                tmem_ld32(tR0 + 32, b);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    w[i] = a[i];
                    w[32 + i] = b[i];
                }
            }
            store_row_sw128(VB, d, w);
            if (tid >= kC) store_row_sw128(AB, tid - kC, row);
            tmem_wait_st();
        }
        tc_fence_before();
        fence_proxy_async();
        __syncthreads();
        // (10) G3: R1 += -(S^T W^T); R0 = S^T Q^T.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id_w = idesc_bf16(128, 64, 0, 1, 1);
            const uint32_t id_q = idesc_bf16(128, 64, 0, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
                umma_bf16(tbase + kColR1, sdesc_sw128(sST + aoff, 16, 1024),
                          sdesc_sw128(sVB + ks * 2048, 8192, 1024), id_w, 1);
            }
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
                const uint32_t boff = kTileBytes + (ks >> 2) * 16384 + (ks & 3) * 32;
                umma_bf16(tbase + kColR0, sdesc_sw128(sST + aoff, 16, 1024),
                          sdesc_sw128(sKQ + boff, 16, 1024), id_q, ks > 0);
            }
            umma_commit(&ms.bar_mma);
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (11) V_new^T -> bf16 operands: plain (ST) and scaled by rr (ST + 16K).
        {
            const int d = tid;
            float vn[64];
            {
                float a[32], b[32];
                tmem_ld32(tR1, a);
                tmem_ld32(tR1 + 32, b);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    vn[i] = a[i];
                    vn[32 + i] = b[i];
                }
            }
            store_row_sw128(ST, d, vn);
#pragma unroll
            for (int t = 0; t < kC; ++t) vn[t] *= ms.rr[t];
            store_row_sw128(ST + 16384, d, vn);
        }
        tc_fence_before();
        fence_proxy_async();
        __syncthreads();
        // (12) G4: R1 = V_new^T intra^T; G5: S^T += (V_new^T o rr) K.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id4 = idesc_bf16(128, 64, 0, 0, 0);
            const uint32_t id5 = idesc_bf16(128, 128, 0, 1, 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tbase + kColR1, sdesc_sw128(sST + ks * 32, 16, 1024),
                          sdesc_sw128(sAB + ks * 32, 16, 1024), id4, ks > 0);
            }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tbase + kColS, sdesc_sw128(sST + 16384 + ks * 32, 16, 1024),
                          sdesc_sw128(sKQ + ks * 2048, 16384, 1024), id5, 1);
            }
            umma_commit(&ms.bar_mma);
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (13) O^T = (Q S)^T diag(cq) + (intra V_new)^T -> bf16 staging [t][d].
        {
            const int d = tid;
            float qs[32], iv[32];
            __nv_bfloat16* OS = reinterpret_cast<__nv_bfloat16*>(VB);
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                tmem_ld32(tR0 + half * 32, qs);
                tmem_ld32(tR1 + half * 32, iv);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int t = half * 32 + i;
                    OS[t * kD + d] = __float2bfloat16_rn(fmaf(qs[i], ms.cq[t], iv[i]));
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        {
            const uint4* src = reinterpret_cast<const uint4*>(VB);
            for (int e = tid; e < valid * 16; e += kThreads) {
                const int t = e >> 4, c = e & 15;
                uint4* dst = reinterpret_cast<uint4*>(out + ((tok0 + t) * p.heads_v + h) * kD) + c;
                *dst = src[e];
            }
        }
        __syncthreads();
        ok = ms.failed == 0;
    }

    // The final state, S^T lane d -> S[:, d].
    if (ok) {
        const int d = tid;
        tc_fence_after();
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
            float x[32];
            tmem_ld32(tS + cb * 32, x);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) state_out[head_state + (cb * 32 + i) * kD + d] = x[i];
        }
    } else if (tid == 0) {
        // Give in-flight copies and MMAs a last bounded chance to land before
        // the TMEM they target is released.
        mbar_wait(&ms.bar_mma, ph_mma, kWaitLimitNs);
        mbar_wait(&ms.bar_tma, ph_tma, kWaitLimitNs);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// [T_total, heads, 128] bf16, boxes of 64 features x 1 head x 64 positions.
bool make_map(CUtensorMap* map, const void* base, int64_t tokens, int heads) {
    auto encode = get_encode();
    if (encode == nullptr) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads),
                                static_cast<cuuint64_t>(tokens > 0 ? tokens : 1)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2,
                                   static_cast<cuuint64_t>(heads) * kD * 2};
    const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kC)};
    const cuuint32_t estride[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Reads and clears the record of a bounded wait that ran out.
cudaError_t take_device_error(int* flag) {
    cudaError_t e = cudaMemcpyFromSymbol(flag, g_tc_error, sizeof(int));
    if (e != cudaSuccess || *flag == 0) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
}

bool chunked_tc_supports(const gdr_params& a) {
    return a.dtype == GDR_DTYPE_BF16 && a.d_k == kD && a.d_v == kD && a.chunk_size == kC;
}

cudaError_t launch_chunked_tc(const Problem& p, const void* q, const void* k, const void* v,
                              const float* g, const float* beta, const float* state_in, void* out,
                              float* state_out, cudaStream_t stream) {
    const uintptr_t align = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                            reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
    if (align & 15) return cudaErrorMisalignedAddress;
    const int64_t tokens = p.cu_seqlens ? p.seq_len : static_cast<int64_t>(p.n_seqs) * p.seq_len;
    if (tokens >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, q, tokens, p.heads_qk) || !make_map(&mk, k, tokens, p.heads_qk) ||
        !make_map(&mv, v, tokens, p.heads_v))
        return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(chunked_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    chunked_tc<<<dim3(p.heads_v, p.n_seqs), kThreads, kSmemBytes, stream>>>(
        p, mq, mk, mv, g, beta, state_in, static_cast<__nv_bfloat16*>(out), state_out);
    return cudaGetLastError();
}

}  // namespace gdr
