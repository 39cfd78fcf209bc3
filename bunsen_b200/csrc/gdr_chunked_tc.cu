// GatedDeltaRule::chunked (delta_rule.rs:223-310) on the sm_100a tensor cores.
//
// bf16 q/k/v, d_k = d_v = 128, chunk C = 64; f32 g, beta, state, f32
// accumulation everywhere. One CTA (256 threads) per (sequence, value head)
// walks the sequence's chunks in order; the state lives in TMEM for the whole
// sequence and touches HBM once on each end. Two CTAs share an SM.
//
// Every contraction of a chunk is one tcgen05.mma group with M = 128 (the
// feature axis, or the 64 keys stacked on the 64 queries), so the tensor
// core always runs full-height tiles. The state is kept transposed,
// S^T [d_v, d_k], so that it is the accumulator of its own update:
//
//   G1  [K;Q] [K;Q]^T       -> TMEM G [128 x 128]  Gram of keys and queries
//        (CUDA cores: norms from its diagonal, decay mask, L =
//         strict_lower(.), intra; A = (I + L)^-1: exact f32 16 x 16 diagonal
//         blocks by forward substitution, off-diagonal blocks by bf16
//         ldmatrix / mma.sync with f32 accumulation)
//   G2  V^T (A diag(beta))^T                -> R1  U^T       [d_v x C]
//       K^T (A diag(beta e^gamma / |k|))^T  -> R0  W^T       [d_k x C]
//        (CUDA cores, while G2 runs: S^T -> bf16 operand, S^T <- e^gamma_C
//         S^T; then W^T -> bf16)
//   G3  R1 += -(S^T W^T)        V_new^T = U^T - (W S)^T
//       S^T Q^T                 -> R0  (Q S)^T
//        (CUDA cores: V_new^T -> bf16, and a copy scaled by e^(gamma_C -
//         gamma_t) / |k_t| per position)
//   G4  V_new^T intra^T         -> R1  (intra V_new)^T
//   G5  S^T += (V_new^T o r) K  the state update
//        (CUDA cores, while the next chunk's tiles load:
//         O^T = (Q S)^T diag(e^gamma / |q| sqrt(d_k)) + R1)
//
// q and k enter the tensor core raw; their L2 norms (delta_rule.rs:112-123)
// and the 1/sqrt(d_k) scale are applied as per-position factors on the
// CUDA-core side, so no pass rewrites the input tiles. Positions past a
// sequence's end take beta = g = 0, which makes them write nothing
// (delta_rule.rs:241-262), whatever the tile holds there.
//
// Threads: warp w serves TMEM lanes 32 (w % 4) .. +31 (one matrix row per
// thread) and column half w / 4 of every 64-column region.
//
// Operand tiles are 128-byte swizzled; TMA writes the input tiles, the
// CUDA-core stages write the rest with the same swizzle. Shared memory:
//   KQ  32 KiB  [k-block][K rows 0-63 | Q rows 64-127] x 128 B  (TMA)
//   VB  16 KiB  V (TMA) -> W^T operand -> V_new^T operand
//   AB  16 KiB  A diag(beta) | A diag(beta e^gamma/|k|) -> (V_new^T o r)
//               operand
//   IN   8 KiB  intra operand
//   ST  36 KiB  L (f32 diagonal blocks, bf16) and the solve's scratch -> S^T
//               operand -> output staging
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gdr_common.cuh"
#include "gdr_decode.cuh"
#include "gdr_sm100.cuh"

namespace gdr {

// Device-side failures since the last gdr_device_error: bit 0, a bounded wait
// ran out; bit 1, a state slot outside the pool.
__device__ int g_tc_error;

namespace {

using namespace sm100;

constexpr int kC = 64;   // chunk
constexpr int kD = 128;  // d_k = d_v
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColG = 128, kColR0 = 128, kColR1 = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

constexpr uint32_t kOffKQ = 0, kOffVB = 32768, kOffAB = 49152, kOffIN = 65536;
constexpr uint32_t kOffST = 73728, kOffMisc = 110592;
constexpr uint32_t kTileBytes = 8192;     // one 64 x 64 bf16 TMA box
constexpr uint32_t kSmemBytes = kOffMisc + 3072 + 1024;  // + alignment slack
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kOsStride = 160;  // bf16 row stride of the output staging tile
constexpr uint32_t kOffZ = 20480;  // in ST: a chunk's z rows [64][128] bf16 (gated norm)
static_assert(kC * kOsStride * 2 <= kOffZ && kOffZ + kC * kD * 2 <= kOffMisc - kOffST,
              "the z rows sit between the output staging and the end of ST");

struct Misc {
    float gam[kC];  // cumulative log decay within the chunk
    float gl[kC];   // the same in log2 units
    float glf[kC];  // gl_t - log2(fk_t): a column's decay and key norm as one exponent
    float bet[kC];  // beta (0 past the end)
    float fk[kC];   // 1 / |k_t|
    float fq[kC];   // 1 / (|q_t| sqrt(d_k))
    float wk[kC];   // beta_t e^gamma_t / |k_t|
    float rr[kC];   // e^(gamma_C - gamma_t) / |k_t|
    float cq[kC];   // e^gamma_t / (|q_t| sqrt(d_k))
    float gstage[2][kC];  // the next chunk's g and beta, landing by cp.async
    uint64_t bar_tma, bar_mma, bar_qs;  // tiles landed; MMA groups; the (Q S)^T group
    uint32_t tmem_base;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&x);
}

__device__ __forceinline__ float lg2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Writes 32 f32 values as bf16 into 16-byte chunks c0 .. c0+3 of a 128-byte
// swizzled row.
__device__ __forceinline__ void store_half_row_sw128(uint8_t* tile, int row, int c0,
                                                     const float* x) {
    uint8_t* base = tile + row * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack_bf16(x[8 * c + 0], x[8 * c + 1]);
        v.y = pack_bf16(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_bf16(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_bf16(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(base + (((c0 + c) ^ (row & 7)) << 4)) = v;
    }
}

// ---- the unit lower-triangular inverse ---------------------------------------
// 64 x 64 bf16 tiles in the 128-byte-swizzled row layout of the MMA operands:
// element (row, col) at row * 128 + ((col / 8) ^ (row % 8)) * 16 + (col % 8) * 2.
__device__ __forceinline__ uint32_t sw_off(int row, int col) {
    return row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Fragments of mma.sync m16n8k16 (bf16 operands, f32 accumulators) for 16 x 16
// blocks of the 64 x 64 swizzled tiles: A (row-major) at (r0, c0) of `tile`,
// B stored [k][n] at (r0, c0); c[nt] covers columns 8 nt .. 8 nt + 7.
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], uint32_t tile, int r0, int c0, int lane) {
    const int i = lane >> 3, j = lane & 7;
    ldsm_x4(a, tile + sw_off(r0 + j + 8 * (i & 1), c0 + 8 * (i >> 1)));
}
__device__ __forceinline__ void frag_b(uint32_t (&b)[4], uint32_t tile, int r0, int c0, int lane) {
    const int i = lane >> 3, j = lane & 7;
    ldsm_x4_trans(b, tile + sw_off(r0 + j + 8 * (i & 1), c0 + 8 * (i >> 1)));
}
// c += A B.
__device__ __forceinline__ void mma16(float (&c)[2][4], const uint32_t (&a)[4],
                                      const uint32_t (&b)[4]) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[nt][0]), "+f"(c[nt][1]), "+f"(c[nt][2]), "+f"(c[nt][3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[2 * nt]), "r"(b[2 * nt + 1]));
}
// An accumulator block as the A operand of the next product (bf16): the
// m16n8 accumulator layout of two column tiles is the m16k16 A layout.
__device__ __forceinline__ void acc_to_a(uint32_t (&a)[4], const float (&c)[2][4]) {
    a[0] = pack_bf16(c[0][0], c[0][1]);
    a[1] = pack_bf16(c[0][2], c[0][3]);
    a[2] = pack_bf16(c[1][0], c[1][1]);
    a[3] = pack_bf16(c[1][2], c[1][3]);
}

// sign * c as bf16 at the 16 x 16 block (r0, c0) of a tile; with `fac`, each
// column scaled by fac[column].
__device__ __forceinline__ void store16_bf16(uint8_t* tile, int r0, int c0, const float (&c)[2][4],
                                             float sign, const float* fac, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        const int col = c0 + 8 * nt + 2 * t;
        const float f0 = fac ? sign * fac[col] : sign, f1 = fac ? sign * fac[col + 1] : sign;
        *reinterpret_cast<uint32_t*>(tile + sw_off(r0 + g, col)) =
            pack_bf16(c[nt][0] * f0, c[nt][1] * f1);
        *reinterpret_cast<uint32_t*>(tile + sw_off(r0 + g + 8, col)) =
            pack_bf16(c[nt][2] * f0, c[nt][3] * f1);
    }
}

// Where the solve's inputs and scratch live (inside the ST region).
constexpr uint32_t kLdStride = 17;                        // f32 diagonal blocks
constexpr uint32_t kOffLd = 0;                            // 4 x 16 x 17 f32
constexpr uint32_t kOffLb = 8192;                         // L, bf16 64 x 64
constexpr uint32_t kOffXb = kOffLb + 8192;                // A, bf16 64 x 64

// A = (I + L)^-1 for the strictly lower 64 x 64 L, in 16 x 16 blocks X_ij:
//  the diagonal blocks X_ii = (I + L_ii)^-1 by exact f32 forward substitution
//  from `Ld` (f32, the four diagonal blocks of L); then, for the two 32 x 32
//  halves lo = {0, 1} and hi = {2, 3}, X_hi,lo = -X_hi L_hi,lo X_lo:
//   step 1  X_10 = -(X_11 L_10) X_00, X_32 = -(X_33 L_32) X_22,
//           X_21 = -(X_22 L_21) X_11, and the parts of P = X_hi L_hi,lo
//           that need only diagonal blocks;
//   step 2  P_3k += X_32 L_2k; X_20, X_30 = -(P_i0 X_00 + P_i1 X_10),
//           X_31 = -P_31 X_11.
//  Products are bf16 mma.sync with f32 accumulation on `Lb` (L in bf16) and
//  `Xb` (the blocks later products read); a product's result feeds the next
//  one from registers, rounded to bf16. Every block of A goes out as it is
//  found, scaled by the column factors fac0 / fac1, to the two G2 operands at
//  AB and AB + kTileBytes, which get their zero blocks above the diagonal
//  here too.
__device__ void unit_lower_inverse_64(uint8_t* ST, int tid, const float* fac0, const float* fac1,
                                      uint8_t* AB) {
    const int warp = tid >> 5, lane = tid & 31;
    const float* Ld = reinterpret_cast<const float*>(ST + kOffLd);
    uint8_t* Xb = ST + kOffXb;
    const uint32_t sLb = smem_u32(ST + kOffLb), sXb = smem_u32(Xb);
    uint8_t* Au = AB;
    uint8_t* Aw = AB + kTileBytes;
    if (tid < 64) {
        const int b = tid >> 4, m = tid & 15;
        const float* Lb = Ld + (16 * b) * kLdStride;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) x[r] = (r == m) ? 1.f : 0.f;
#pragma unroll
        for (int s = 0; s < 15; ++s)
#pragma unroll
            for (int r = s + 1; r < 16; ++r) x[r] = fmaf(-Lb[r * kLdStride + s], x[s], x[r]);
        const int col = 16 * b + m;
        const float f0 = fac0[col], f1 = fac1[col];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const uint32_t off = sw_off(16 * b + r, col);
            *reinterpret_cast<__nv_bfloat16*>(Xb + off) = __float2bfloat16_rn(x[r]);
            *reinterpret_cast<__nv_bfloat16*>(Au + off) = __float2bfloat16_rn(x[r] * f0);
            *reinterpret_cast<__nv_bfloat16*>(Aw + off) = __float2bfloat16_rn(x[r] * f1);
        }
    } else {
        // The six blocks above the block diagonal of both G2 operands are zero:
        // 6 blocks x 16 rows x 2 16-byte chunks x 2 operands.
        for (int e = tid - 64; e < 6 * 16 * 2 * 2; e += kThreads - 64) {
            const int blk = e >> 6, r = (e >> 2) & 15, half = (e >> 1) & 1, mtx = e & 1;
            const int ib = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
            const int jb = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
            const int row = 16 * ib + r, col = 16 * jb + 8 * half;
            *reinterpret_cast<uint4*>((mtx ? Aw : Au) + sw_off(row, col)) = make_uint4(0, 0, 0, 0);
        }
    }
    __syncthreads();
    auto put = [&](int i, int j, const float (&c)[2][4], bool keep) {  // X_ij = -c
        if (keep) store16_bf16(Xb, 16 * i, 16 * j, c, -1.f, nullptr, lane);
        store16_bf16(Au, 16 * i, 16 * j, c, -1.f, fac0, lane);
        store16_bf16(Aw, 16 * i, 16 * j, c, -1.f, fac1, lane);
    };
    uint32_t a[4], b[4];
    float p0[2][4] = {}, p1[2][4] = {};  // P_i0, P_i1 of warps 3 .. 5
    if (warp < 3) {
        // Step 1: X_10 (warp 0), X_32 (warp 1), X_21 (warp 2) = -(X_ii L_ij) X_jj.
        const int i = warp == 0 ? 1 : (warp == 1 ? 3 : 2), j = i - 1;
        frag_a(a, sXb, 16 * i, 16 * i, lane);
        frag_b(b, sLb, 16 * i, 16 * j, lane);
        mma16(p0, a, b);
        acc_to_a(a, p0);
        frag_b(b, sXb, 16 * j, 16 * j, lane);
        float x[2][4] = {};
        mma16(x, a, b);
        put(i, j, x, warp < 2);  // X_10 and X_32 are read by step 2
    } else if (warp < 6) {
        // Step 1: P_20, P_21 = X_22 L_2k (warp 3); P_30, P_31 (warp 4) and
        // P_31 (warp 5) start as X_33 L_3k.
        const int i = warp == 3 ? 2 : 3;
        frag_a(a, sXb, 16 * i, 16 * i, lane);
        if (warp < 5) {
            frag_b(b, sLb, 16 * i, 0, lane);
            mma16(p0, a, b);
        }
        frag_b(b, sLb, 16 * i, 16, lane);
        mma16(p1, a, b);
    }
    __syncthreads();
    if (warp >= 3 && warp < 6) {
        // Step 2.
        if (warp > 3) {  // P_3k += X_32 L_2k
            frag_a(a, sXb, 48, 32, lane);
            if (warp == 4) {
                frag_b(b, sLb, 32, 0, lane);
                mma16(p0, a, b);
            }
            frag_b(b, sLb, 32, 16, lane);
            mma16(p1, a, b);
        }
        float x[2][4] = {};
        if (warp < 5) {  // P_i0 X_00
            acc_to_a(a, p0);
            frag_b(b, sXb, 0, 0, lane);
            mma16(x, a, b);
        }
        acc_to_a(a, p1);  // P_i1 X_10 (X_20, X_30) or P_31 X_11 (X_31)
        frag_b(b, sXb, 16, warp == 5 ? 16 : 0, lane);
        mma16(x, a, b);
        put(warp == 3 ? 2 : 3, warp == 5 ? 1 : 0, x, false);
    }
}

// Variants of an item, for the segments of a split sequence: start from the
// identity instead of state_in; take v as zero (no V tiles, U = 0); write no
// output (no Q tiles, no output products).
constexpr uint32_t kItemIdentity = 1, kItemZeroV = 2, kItemNoOut = 4;

// One (sequence, value head): positions [t0, t0 + len) of value head h, from
// state_in (null: zeros; may equal state_out) to state_out (null: not
// stored), both that head's [d_k, d_v] f32 state. `smem` is the CTA's
// 1024-aligned dynamic shared memory; `tbase` the CTA's 256 TMEM columns
// (tmem_acquire). kFlags: kItem* above.
template <uint32_t kFlags = 0>
__device__ __forceinline__ void prefill_item(const Problem& p, const CUtensorMap* tm_q,
                                             const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                             const float* __restrict__ g,
                                             const float* __restrict__ beta,
                                             __nv_bfloat16* __restrict__ out, int64_t t0,
                                             int64_t len, int h, const float* state_in,
                                             float* state_out, uint8_t* smem, uint32_t tbase) {
    constexpr bool zero_v = kFlags & kItemZeroV, with_out = !(kFlags & kItemNoOut);
    uint8_t* KQ = smem + kOffKQ;
    uint8_t* VB = smem + kOffVB;
    uint8_t* AB = smem + kOffAB;
    uint8_t* IN = smem + kOffIN;
    uint8_t* ST = smem + kOffST;
    Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qd = warp & 3, hf = warp >> 2;
    const int row = 32 * qd + lane;  // this thread's TMEM lane
    const int hq = h / p.group;
    const int n_chunks = static_cast<int>((len + kC - 1) / kC);

    if (tid == 0) {
        mbar_init(&ms.bar_tma, 1);
        mbar_init(&ms.bar_mma, 1);
        mbar_init(&ms.bar_qs, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(qd * 32) << 16);
    // Operand descriptors; a tile offset is added to the start-address field.
    const uint64_t dKQ = sdesc_sw128(smem_u32(KQ), 16, 1024);      // K-major K, Q
    const uint64_t dKQmn = sdesc_sw128(smem_u32(KQ), 16384, 1024);  // MN-major K
    const uint64_t dVBmn = sdesc_sw128(smem_u32(VB), 8192, 1024);   // MN-major V, W^T
    const uint64_t dAB = sdesc_sw128(smem_u32(AB), 16, 1024);
    const uint64_t dIN = sdesc_sw128(smem_u32(IN), 16, 1024);
    const uint64_t dST = sdesc_sw128(smem_u32(ST), 16, 1024);
    const uint64_t dVB = sdesc_sw128(smem_u32(VB), 16, 1024);       // K-major V_new^T
    auto at = [](uint64_t d, uint32_t off) { return d + (off >> 4); };

    // Thread 0: chunk ci's K, Q, V tiles (without an output, Q rows of the
    // Gram are never read; with v zero, V is not read).
    const uint32_t tile_tx = (2 + (with_out ? 2 : 0) + (zero_v ? 0 : 2)) * kTileBytes;
    auto issue_tiles = [&](int ci) {
        fence_proxy_async();
        mbar_expect_tx(&ms.bar_tma, tile_tx);
        const int tok = static_cast<int>(t0 + static_cast<int64_t>(ci) * kC);
        tma_load_3d(KQ + 0 * kTileBytes, tm_k, &ms.bar_tma, 0, hq, tok);
        tma_load_3d(KQ + 2 * kTileBytes, tm_k, &ms.bar_tma, 64, hq, tok);
        if constexpr (with_out) {
            tma_load_3d(KQ + 1 * kTileBytes, tm_q, &ms.bar_tma, 0, hq, tok);
            tma_load_3d(KQ + 3 * kTileBytes, tm_q, &ms.bar_tma, 64, hq, tok);
        }
        if constexpr (!zero_v) {
            tma_load_3d(VB + 0 * kTileBytes, tm_v, &ms.bar_tma, 0, h, tok);
            tma_load_3d(VB + 1 * kTileBytes, tm_v, &ms.bar_tma, 64, h, tok);
        }
    };
    auto prefetch_tiles = [&](int ci) {  // one thread: chunk ci's tiles into L2
        const int tok = static_cast<int>(t0 + static_cast<int64_t>(ci) * kC);
        tma_prefetch_3d(tm_k, 0, hq, tok);
        tma_prefetch_3d(tm_k, 64, hq, tok);
        if constexpr (with_out) {
            tma_prefetch_3d(tm_q, 0, hq, tok);
            tma_prefetch_3d(tm_q, 64, hq, tok);
        }
        if constexpr (!zero_v) {
            tma_prefetch_3d(tm_v, 0, h, tok);
            tma_prefetch_3d(tm_v, 64, h, tok);
        }
    };
    // Threads 0..127: chunk ci's g (tid < 64) or beta into ms.gstage by 4-byte
    // cp.async (zero-filled past the end), so no register waits for them.
    // With the layer's gates fused, the 4-byte word holding the projection a
    // (or b) is staged instead and put_gates turns it into g (or beta).
    auto stage_gates = [&](int ci) {
        const int t = tid & (kC - 1), which = tid >> 6;
        const int64_t pos = static_cast<int64_t>(ci) * kC + t;
        const int64_t at = pos < len ? pos : len - 1;
        const int64_t i = (t0 + at) * p.heads_v + h;
        const void* src;
        if (p.gate_a == nullptr)
            src = (which ? beta : g) + i;
        else if (p.gate_bf16)
            src = static_cast<const uint8_t*>(which ? p.gate_b : p.gate_a) + ((2 * i) & ~int64_t{3});
        else
            src = static_cast<const float*>(which ? p.gate_b : p.gate_a) + i;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(
                         smem_u32(&ms.gstage[which][t])),
                     "l"(src), "r"(pos < len ? 4 : 0)
                     : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto gates_landed = [] { asm volatile("cp.async.wait_group 0;" ::: "memory"); };
    // Threads 0..127, after their own copy landed: with the layer's gates
    // fused, chunk ci's staged projection word becomes g (tid < 64) or beta,
    // zero past the end (as the zero-filled g and beta are).
    auto convert_gates = [&](int ci) {
        if (p.gate_a == nullptr) return;
        const int t = tid & (kC - 1), which = tid >> 6;
        const int64_t pos = static_cast<int64_t>(ci) * kC + t;
        float x = ms.gstage[which][t];
        if (p.gate_bf16) {
            const int64_t i = (t0 + (pos < len ? pos : len - 1)) * p.heads_v + h;
            x = __uint_as_float((__float_as_uint(x) >> ((i & 1) ? 16 : 0)) << 16);
        }
        ms.gstage[which][t] = pos >= len ? 0.f
                              : which   ? gate_beta(x, p.gate_dtype)
                                        : gate_g(x, p.a_log[h], p.dt_bias[h]);
    };
    // Warp 0: the staged gates into the chunk's arrays, the log decay as its
    // running sum (positions 2 lane, 2 lane + 1).
    auto put_gates = [&] {
        const float pg0 = ms.gstage[0][2 * lane], pg1 = ms.gstage[0][2 * lane + 1];
        const float pb0 = ms.gstage[1][2 * lane], pb1 = ms.gstage[1][2 * lane + 1];
        float incl = pg0 + pg1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const float g0 = incl - pg1, g1 = incl;
        ms.gam[2 * lane] = g0;
        ms.gam[2 * lane + 1] = g1;
        ms.gl[2 * lane] = g0 * kLog2e;
        ms.gl[2 * lane + 1] = g1 * kLog2e;
        ms.bet[2 * lane] = pb0;
        ms.bet[2 * lane + 1] = pb1;
    };

    if (tid == 0 && n_chunks > 0) issue_tiles(0);
    if (tid == kThreads - 32 && n_chunks > 1) prefetch_tiles(1);
    if (tid < 2 * kC && n_chunks > 0) {
        stage_gates(0);
        gates_landed();
        convert_gates(0);
    }
    __syncthreads();
    if (warp == 0 && n_chunks > 0) put_gates();

    // The initial state, transposed into TMEM: lane d holds S[:, d].
    {
        constexpr bool identity = kFlags & kItemIdentity;
#pragma unroll 1
        for (int cb = 0; cb < 2; ++cb) {
            float x[32];
            const int c0 = 64 * hf + 32 * cb;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                x[i] = identity   ? (c0 + i == row ? 1.f : 0.f)
                       : state_in ? state_in[(c0 + i) * kD + row]
                                  : 0.f;
            tmem_st32(lane_addr + kColS + c0, x);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();

    uint32_t ph_tma = 0, ph_mma = 0, ph_qs = 0;
    auto issue_g1 = [&] {  // thread 0, once the chunk's tiles have landed
        tc_fence_after();
        // Without an output only the keys' Gram (columns 0-63) is read.
        const uint32_t id = idesc_bf16(128, with_out ? 128 : 64, 0, 0, 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma_bf16(tbase + kColG, at(dKQ, off), at(dKQ, off), id, ks > 0);
        }
        umma_commit(&ms.bar_mma);
    };
    // A wait that runs out marks this thread; the CTA learns of it at the
    // next __syncthreads_or, so every thread leaves the loop together.
    int fail = 0;
    auto wait = [&](uint64_t* bar, uint32_t& ph) {
        if (!mbar_wait(bar, ph, kWaitLimitNs)) {
            fail = 1;
            atomicOr(&g_tc_error, 1);
        }
        ph ^= 1u;
    };

#pragma unroll 1
    for (int ci = 0; ci < n_chunks; ++ci) {
        const int64_t tok0 = t0 + static_cast<int64_t>(ci) * kC;
        const int64_t left = len - static_cast<int64_t>(ci) * kC;
        const int valid = static_cast<int>(left < kC ? left : kC);
        // (b)+(c) The tiles (this chunk's gates are in shared memory), then
        //       G1: [K;Q] [K;Q]^T -> G. After the first chunk, G1 was issued
        //       at the end of the previous chunk.
        if (ci == 0) {
            wait(&ms.bar_tma, ph_tma);
            if (tid == 0) issue_g1();
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (e) This thread's 32 Gram columns, and the norms from the diagonal.
        float gr[32];
        tmem_ld32(lane_addr + kColG + 32 * hf, gr);
        if (with_out && qd >= 2 && hf == 0) {
            float dq[32];
            tmem_ld32(lane_addr + kColG + 32 * qd, dq);  // q_i . q_i at column 64 + i
            tmem_wait_ld();
            float d = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) d = (j == lane) ? dq[j] : d;
            ms.fq[row - kC] = l2_factor(p, d) * p.q_scale;
        }
        tmem_wait_ld();
        if (qd < 2 && hf == qd) {
            float d = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) d = (j == lane) ? gr[j] : d;
            const float fk = l2_factor(p, d);
            ms.fk[row] = fk;
            ms.glf[row] = ms.gl[row] - lg2(fk);
        }
        tc_fence_before();
        // Every thread is past the previous chunk's output (its staging reads
        // end before (f) writes ST), and a failure anywhere ends the loop.
        if (__syncthreads_or(fail)) break;
        // (f) Per-position factors; rows of L (f32) and of intra (bf16 operand).
        const float decay = __expf(ms.gam[kC - 1]);
        if (tid < kC) {
            const float gt = ms.gam[tid], last = ms.gam[kC - 1];
            const float eg = __expf(gt);
            ms.wk[tid] = ms.bet[tid] * eg * ms.fk[tid];
            ms.rr[tid] = __expf(last - gt) * ms.fk[tid];
            if constexpr (with_out) ms.cq[tid] = eg * ms.fq[tid];
        }
        if (with_out || qd < 2) {  // without an output, no intra rows
            const bool key_row = qd < 2;
            const int i = key_row ? row : row - kC;
            // This warp's 32 x 32 block of rows (i) and columns (j): below the
            // diagonal, on it, or above it (all zero) -- uniform per warp.
            const int rblk = key_row ? qd : qd - 2;
            float v[32];
            if (rblk < hf) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = 0.f;
            } else {
                // rowf_i fk_j e^(gamma_i - gamma_j) = 2^(a_i - glf_j): one
                // exponential carries the decay and both norm factors.
                const float rowf = key_row ? ms.bet[i] * ms.fk[i] : ms.fq[i];
                const float a = ms.gl[i] + lg2(rowf);
                const int lim = key_row ? i : i + 1;  // j < lim survives
                const float4* glf4 = reinterpret_cast<const float4*>(ms.glf + 32 * hf);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 b = glf4[c];
                    v[4 * c + 0] = gr[4 * c + 0] * ex2(a - b.x);
                    v[4 * c + 1] = gr[4 * c + 1] * ex2(a - b.y);
                    v[4 * c + 2] = gr[4 * c + 2] * ex2(a - b.z);
                    v[4 * c + 3] = gr[4 * c + 3] * ex2(a - b.w);
                }
                if (rblk == hf) {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) v[jj] = (32 * hf + jj < lim) ? v[jj] : 0.f;
                }
            }
            if (key_row) {
                // L in bf16 for the solve's products; its diagonal 16 x 16
                // block in f32 for the exact forward substitution.
                store_half_row_sw128(ST + kOffLb, i, 4 * hf, v);
                if (rblk == hf) {
                    float* ld = reinterpret_cast<float*>(ST + kOffLd) + i * kLdStride;
                    const bool upper = (i >> 4) & 1;
#pragma unroll
                    for (int s2 = 0; s2 < 16; ++s2) ld[s2] = upper ? v[16 + s2] : v[s2];
                }
            } else {
                store_half_row_sw128(IN, i, 4 * hf, v);
            }
        }
        __syncthreads();
        // (g) A = (I + L)^-1. Meanwhile the chunk after next warms L2.
        if (tid == kThreads - 32 && ci + 2 < n_chunks) prefetch_tiles(ci + 2);
        unit_lower_inverse_64(ST, tid, ms.bet, ms.wk, AB);
        fence_proxy_async();
        __syncthreads();
        // (i) G2: U^T = V^T Au^T -> R1; W^T = K^T Aw^T -> R0.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id = idesc_bf16(128, 64, 1, 0, 0);
            if constexpr (!zero_v) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma_bf16(tbase + kColR1, at(dVBmn, ks * 2048), at(dAB, ks * 32), id, ks > 0);
            }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                umma_bf16(tbase + kColR0, at(dKQmn, ks * 2048), at(dAB, kTileBytes + ks * 32),
                          id, ks > 0);
            umma_commit(&ms.bar_mma);
        }
        // The next chunk's gates start loading (they are published in (p)).
        if (tid < 2 * kC && ci + 1 < n_chunks) stage_gates(ci + 1);
        // (j) While G2 runs: S^T -> bf16 operand; S^T <- e^gamma_C S^T.
        {
#pragma unroll 1
            for (int cb = 0; cb < 2; ++cb) {
                float x[32];
                const uint32_t col = kColS + 64 * hf + 32 * cb;
                tmem_ld32(lane_addr + col, x);
                tmem_wait_ld();
                store_half_row_sw128(ST + hf * 16384, row, 4 * cb, x);
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] *= decay;
                tmem_st32(lane_addr + col, x);
            }
            tmem_wait_st();
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (l) W^T -> bf16 MN-major operand (over V, which G2 consumed).
        {
            float w[32];
            tmem_ld32(lane_addr + kColR0 + 32 * hf, w);
            tmem_wait_ld();
            store_half_row_sw128(VB, row, 4 * hf, w);
        }
        tc_fence_before();
        fence_proxy_async();
        __syncthreads();
        // (m) G3: R1 += -(S^T W^T) (R1 = -(S^T W^T) when U = 0), issued by
        //     thread 0 and committed alone so (n) starts while R0 = S^T Q^T
        //     runs; that half is issued by thread 32 (committed to bar_qs), so
        //     neither issuing thread waits on the other's MMAs.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id_w = idesc_bf16(128, 64, 0, 1, 1);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
                umma_bf16(tbase + kColR1, at(dST, aoff), at(dVBmn, ks * 2048), id_w,
                          !zero_v || ks > 0);
            }
            umma_commit(&ms.bar_mma);
        } else if (tid == 32) {
            tc_fence_after();
            const uint32_t id_q = idesc_bf16(128, 64, 0, 0, 0);
            if constexpr (with_out) {
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
                    const uint32_t boff = kTileBytes + (ks >> 2) * 16384 + (ks & 3) * 32;
                    umma_bf16(tbase + kColR0, at(dST, aoff), at(dKQ, boff), id_q, ks > 0);
                }
            }
            umma_commit(&ms.bar_qs);
        }
        wait(&ms.bar_mma, ph_mma);
        tc_fence_after();
        // (n) V_new^T -> bf16 operands: plain (VB, free since G3's first
        //     group) and scaled by rr (AB, free since G2); ST is still read by
        //     the (Q S)^T group.
        {
            float vn[32];
            tmem_ld32(lane_addr + kColR1 + 32 * hf, vn);
            tmem_wait_ld();
            store_half_row_sw128(VB, row, 4 * hf, vn);
            const float4* rr4 = reinterpret_cast<const float4*>(ms.rr + 32 * hf);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 r = rr4[c];
                vn[4 * c] *= r.x;
                vn[4 * c + 1] *= r.y;
                vn[4 * c + 2] *= r.z;
                vn[4 * c + 3] *= r.w;
            }
            store_half_row_sw128(AB, row, 4 * hf, vn);
        }
        if (tid < 2 * kC) {
            gates_landed();
            if (ci + 1 < n_chunks) convert_gates(ci + 1);
        }
        tc_fence_before();
        fence_proxy_async();
        __syncthreads();
        // (o) G4: R1 = V_new^T intra^T; G5: S^T += (V_new^T o rr) K.
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id4 = idesc_bf16(128, 64, 0, 0, 0);
            const uint32_t id5 = idesc_bf16(128, 128, 0, 1, 0);
            if constexpr (with_out) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    umma_bf16(tbase + kColR1, at(dVB, ks * 32), at(dIN, ks * 32), id4, ks > 0);
            }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                umma_bf16(tbase + kColS, at(dAB, ks * 32), at(dKQmn, ks * 2048), id5, 1);
            umma_commit(&ms.bar_mma);
        }
        // (p) The next chunk's gates (this chunk's are no longer read).
        if (warp == 0 && ci + 1 < n_chunks) put_gates();
        wait(&ms.bar_mma, ph_mma);
        wait(&ms.bar_qs, ph_qs);
        tc_fence_after();
        // (r) The next chunk's tiles load while this chunk's output is written.
        //     With the gated norm, this chunk's z rows land in the tail of ST
        //     (free once the Q S group is done), each thread copying the row
        //     pieces it normalises in (s).
        if (tid == 0 && ci + 1 < n_chunks) issue_tiles(ci + 1);
        // Warp 0 issues the next chunk's G1 and leaves the output rows to the
        // other warps (`lead` threads skipped), here and in (s).
        const int lead = ci + 1 < n_chunks ? 32 : 0;
        if (with_out && p.norm_z != nullptr) {
            for (int e = tid - lead; e >= 0 && e < kC * 16; e += kThreads - lead) {
                const int t = e >> 4, c = e & 15;
                const int tt = t < valid ? t : 0;
                const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(p.norm_z) +
                                           ((tok0 + tt) * p.heads_v + h) * kD + 8 * c;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                                 smem_u32(ST + kOffZ + t * 256 + 16 * c)),
                             "l"(src), "r"(t < valid ? 16 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        // (s) O^T = (Q S)^T diag(cq) + (intra V_new)^T -> bf16 staging [t][d].
        if constexpr (with_out) {
            float qs[32], iv[32];
            tmem_ld32(lane_addr + kColR0 + 32 * hf, qs);
            tmem_ld32(lane_addr + kColR1 + 32 * hf, iv);
            tmem_wait_ld();
            const float4* cq4 = reinterpret_cast<const float4*>(ms.cq + 32 * hf);
            float o[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 q = cq4[c];
                o[4 * c] = fmaf(qs[4 * c], q.x, iv[4 * c]);
                o[4 * c + 1] = fmaf(qs[4 * c + 1], q.y, iv[4 * c + 1]);
                o[4 * c + 2] = fmaf(qs[4 * c + 2], q.z, iv[4 * c + 2]);
                o[4 * c + 3] = fmaf(qs[4 * c + 3], q.w, iv[4 * c + 3]);
            }
            // Lanes 2m and 2m+1 hold features d, d+1 of every position: swap
            // so that the even lane stores (t, d..d+1) for even t and the odd
            // lane for odd t, as 32-bit words of the [t][d] staging tile.
            uint32_t* OS = reinterpret_cast<uint32_t*>(ST);
            const bool odd = lane & 1;
            const int d0 = row & ~1;
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const float send = odd ? o[i] : o[i + 1];
                const float got = __shfl_xor_sync(0xffffffffu, send, 1);
                const int t = 32 * hf + i + (odd ? 1 : 0);
                const uint32_t w = odd ? pack_bf16(got, o[i + 1]) : pack_bf16(o[i], got);
                OS[t * (kOsStride / 2) + (d0 >> 1)] = w;
            }
        }
        tc_fence_before();
        __syncthreads();
        // R0 and R1 have been read: the next chunk's G1 (its tiles were issued
        // at (r)) runs while this chunk's output is stored.
        if (ci + 1 < n_chunks) {
            if (tid == 0) {
                wait(&ms.bar_tma, ph_tma);
                issue_g1();
            } else {
                ph_tma ^= 1u;
            }
        }
        if constexpr (with_out) {
            if (p.norm_z == nullptr) {
                for (int e = tid - lead; e >= 0 && e < valid * 16; e += kThreads - lead) {
                    const int t = e >> 4, c = e & 15;
                    const uint4* src = reinterpret_cast<const uint4*>(ST + t * kOsStride * 2) + c;
                    uint4* dst =
                        reinterpret_cast<uint4*>(out + ((tok0 + t) * p.heads_v + h) * kD) + c;
                    *dst = *src;
                }
            } else {
                // The layer's gated RMS norm of each output row: 16 lanes hold
                // a row's 128 features (8 each) and reduce over them; z from
                // the rows staged at (r).
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                // The loop below ends in full-warp shuffles, so every lane of
                // a warp must run it equally often: kC * 16, kThreads and
                // `lead` (0 or 32) are all multiples of the warp size.
                static_assert((kC * 16) % 32 == 0 && kThreads % 32 == 0,
                              "whole warps walk the output rows");
                const int cw = tid & 15;
                const float4 w0 = reinterpret_cast<const float4*>(p.norm_w)[2 * cw];
                const float4 w1 = reinterpret_cast<const float4*>(p.norm_w)[2 * cw + 1];
                const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll 1
                for (int e = tid - lead; e >= 0 && e < kC * 16; e += kThreads - lead) {
                    const int t = e >> 4, c = e & 15;
                    const bool in = t < valid;
                    const uint4 src = reinterpret_cast<const uint4*>(ST + t * kOsStride * 2)[c];
                    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&src);
                    float x[8], ss = 0.f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        x[j] = __bfloat162float(xb[j]);
                        ss = fmaf(x[j], x[j], ss);
                    }
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                    if (in) {
                        const float r = rsqrtf(ss / kD + p.norm_eps);
                        const int64_t row = ((tok0 + t) * p.heads_v + h) * kD + 8 * c;
                        const uint4 zv = *reinterpret_cast<const uint4*>(ST + kOffZ + t * 256 + 16 * c);
                        const __nv_bfloat16* zb = reinterpret_cast<const __nv_bfloat16*>(&zv);
                        uint4 y;
                        uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float s0 = silu(__bfloat162float(zb[2 * j]));
                            const float s1 = silu(__bfloat162float(zb[2 * j + 1]));
                            yw[j] = pack_bf16(x[2 * j] * r * wv[2 * j] * s0,
                                              x[2 * j + 1] * r * wv[2 * j + 1] * s1);
                        }
                        *reinterpret_cast<uint4*>(out + row) = y;
                    }
                }
            }
        }
    }
    const bool ok = !__syncthreads_or(fail);

    // The final state, S^T lane d -> S[:, d].
    if (ok) {
        tc_fence_after();
        if (state_out != nullptr) {
#pragma unroll 1
            for (int cb = 0; cb < 2; ++cb) {
                float x[32];
                const int c0 = 64 * hf + 32 * cb;
                tmem_ld32(lane_addr + kColS + c0, x);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) state_out[(c0 + i) * kD + row] = x[i];
            }
        }
    } else if (tid == 0) {
        // Give in-flight copies and MMAs a last bounded chance to land before
        // the TMEM and shared memory they target are used again.
        mbar_wait(&ms.bar_mma, ph_mma, kWaitLimitNs);
        mbar_wait(&ms.bar_qs, ph_qs, kWaitLimitNs);
        mbar_wait(&ms.bar_tma, ph_tma, kWaitLimitNs);
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // the barriers may be initialised again by the next item
        mbar_inval(&ms.bar_tma);
        mbar_inval(&ms.bar_mma);
        mbar_inval(&ms.bar_qs);
    }
}

// The CTA's 256 TMEM columns, allocated once by warp 0, which then gives up
// the CTA's right to allocate again (a CTA allocates exactly once, so the SM
// never holds a request back); every thread gets the base address. Items
// reuse the columns; tmem_release frees them when the CTA is done.
__device__ __forceinline__ uint32_t tmem_acquire(uint8_t* smem) {
    Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);
    if ((threadIdx.x >> 5) == 0) {
        tmem_alloc(&ms.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t base = ms.tmem_base;
    __syncthreads();
    return base;
}

__device__ __forceinline__ void tmem_release(uint32_t tbase) {
    tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 0) tmem_dealloc(tbase, kTmemCols);
}

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                      ~static_cast<uintptr_t>(1023));
}

// Packs of at most this many sequences run longest first.
constexpr int kRankMax = 128;

// The sequence of rank y when a packed batch's sequences are ordered by
// length, longest first (ties by index). Every thread gets the answer.
__device__ int longest_first(const Problem& p, int y, uint8_t* scratch) {
    int* lens = reinterpret_cast<int*>(scratch);
    int* pick = lens + kRankMax;
    const int n = p.n_seqs;
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        int64_t a, b;
        seq_span(p, s, a, b);
        lens[s] = static_cast<int>(b - a);
    }
    if (threadIdx.x == 0) *pick = y;
    __syncthreads();
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        const int ls = lens[s];
        int rank = 0;
        for (int u = 0; u < n; ++u) rank += (lens[u] > ls) || (lens[u] == ls && u < s);
        if (rank == y) *pick = s;
    }
    __syncthreads();
    const int s = *pick;
    __syncthreads();
    return s;
}

__global__ void __launch_bounds__(kThreads, 2)
chunked_tc(const Problem p, const __grid_constant__ CUtensorMap tm_q,
           const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
           const float* __restrict__ g, const float* __restrict__ beta, const float* state_in,
           __nv_bfloat16* __restrict__ out, float* state_out) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    const int h = blockIdx.x, y = blockIdx.y;
    const int s = (p.cu_seqlens != nullptr && p.n_seqs <= kRankMax)
                      ? longest_first(p, y, smem + kOffST)
                      : y;
    int64_t t0, t1;
    seq_span(p, s, t0, t1);
    const int64_t hs = (static_cast<int64_t>(s) * p.heads_v + h) * kD * kD;
    const uint32_t tbase = tmem_acquire(smem);
    prefill_item(p, &tm_q, &tm_k, &tm_v, g, beta, out, t0, t1 - t0, h,
                 state_in ? state_in + hs : nullptr, state_out + hs, smem, tbase);
    tmem_release(tbase);
}

// The work list of a continuous batch, built in the caller's workspace:
// work[0] = prefill sequences (length > 1), work[1] = decode rows (length 1),
// work[2], work[3] = the two queues' cursors (zeroed here), work[4] = how
// many of the `grid` CTAs start on the prefill queue, then (from
// work[kWorkHeader]) the sequence indices, prefill ones first by decreasing
// chunk count, then the decode rows. One CTA of 1024 threads; sequences of
// length 0 are left out.
//
// The prefill share of the grid follows the work: a (prefill chunk, head)
// item costs about kChunkCost and a (decode row, head) item about kRowCost
// in CTA-time (a chunk's dependent MMA and CUDA-core stages, against a
// 128 KiB state round trip sharing HBM). On B200, 8 x 2048 prefill tokens
// with 1024 decode rows (32 value heads) run in 0.94-0.95 ms for any ratio
// from 2.0 to 5.5 and in 1.06-1.10 ms below 1.6, where the prefill queue
// needs one more round of items; 2.5 sits inside the flat range. A share that
// would run the prefill items in more than one round is raised to the CTAs
// for one round fewer: half that batch (4 segments, 512 rows) went from 0.564
// to 0.492 ms, the full one stayed at 0.94 ms.
constexpr int kPlanBuckets = 1024;
constexpr int kWorkHeader = 8;
constexpr float kChunkCost = 2.5f, kRowCost = 1.0f;
__global__ void __launch_bounds__(1024)
plan_mixed(const Problem p, int32_t* work, int grid) {
    __shared__ int hist[kPlanBuckets];
    __shared__ int n_pre, n_dec;
    __shared__ unsigned long long chunks;
    const int n = p.n_seqs;
    auto bucket = [&](int64_t len) {  // descending chunk count
        const int64_t c = (len + kC - 1) / kC;
        return kPlanBuckets - 1 - static_cast<int>(c < kPlanBuckets - 1 ? c : kPlanBuckets - 1);
    };
    for (int i = threadIdx.x; i < kPlanBuckets; i += blockDim.x) hist[i] = 0;
    if (threadIdx.x == 0) {
        n_pre = n_dec = 0;
        chunks = 0;
    }
    __syncthreads();
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        int64_t a, b;
        seq_span(p, s, a, b);
        if (b - a > 1) {
            atomicAdd(&hist[bucket(b - a)], 1);
            atomicAdd(&n_pre, 1);
            atomicAdd(&chunks, static_cast<unsigned long long>((b - a + kC - 1) / kC));
        } else if (b - a == 1) {
            atomicAdd(&n_dec, 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the buckets into cursors
        int acc = 0;
        for (int i = 0; i < kPlanBuckets; ++i) {
            const int c = hist[i];
            hist[i] = acc;
            acc += c;
        }
        work[0] = n_pre;
        work[1] = n_dec;
        work[2] = 0;
        work[3] = 0;
        const float wp = kChunkCost * static_cast<float>(chunks);
        const float wd = kRowCost * static_cast<float>(n_dec);
        int pre_ctas = n_pre == 0 ? 0
                       : n_dec == 0 ? grid
                                    : static_cast<int>(ceilf(grid * wp / (wp + wd)));
        if (pre_ctas > 0 && n_dec > 0) {
            // Prefill items hold their CTA for a whole chain: when the share
            // would run them in r > 1 rounds, give the queue the CTAs for one
            // round fewer (freed CTAs move to the decode rows).
            const int64_t items = static_cast<int64_t>(n_pre) * p.heads_v;
            const int64_t rounds = (items + pre_ctas - 1) / pre_ctas;
            if (rounds > 1) {
                const int64_t fewer = (items + rounds - 2) / (rounds - 1);
                if (fewer <= grid) pre_ctas = static_cast<int>(fewer);
            }
        }
        work[4] = pre_ctas < grid ? pre_ctas : grid;
        n_dec = n_pre;  // cursor of the decode rows
    }
    __syncthreads();
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        int64_t a, b;
        seq_span(p, s, a, b);
        if (b - a > 1)
            work[kWorkHeader + atomicAdd(&hist[bucket(b - a)], 1)] = s;
        else if (b - a == 1)
            work[kWorkHeader + atomicAdd(&n_dec, 1)] = s;
    }
}

// A continuous batch, persistent: each CTA pulls (sequence, value head) items
// from two queues in the work list -- prefill segments through prefill_item,
// decode rows through the CUDA-core recurrent body -- until both are empty.
// The first work[4] CTAs start on the prefill queue (longest segments first)
// and the rest on the decode rows, in proportion to the two queues' work, so
// the latency-bound prefill does not hold the slots the bandwidth-bound decode
// rows need; a CTA whose queue runs dry moves to the other.
//
// Decode rows are pipelined: while one row's state is updated in registers
// and written back, the next row's 64 KiB state is already on its way into
// shared memory by a bulk copy.
constexpr uint32_t kOffDecStage = 16384;                      // 64 KiB staging
constexpr uint32_t kOffDecBar = kOffDecStage + kD * kD * 4;   // its mbarrier

struct MixedItem {
    int qn, s, h;  // queue (0 prefill, 1 decode), sequence, value head
    float* st;     // the head's state in the pool
};

__global__ void __launch_bounds__(kThreads, 2)
mixed_tc(const Problem p, const __grid_constant__ CUtensorMap tm_q,
         const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
         const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
         const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
         const float* __restrict__ beta, float* pool, const int32_t* slots, int32_t n_slots,
         __nv_bfloat16* __restrict__ out, int32_t* work) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    __shared__ MixedItem shared_item;
    const uint32_t tbase = tmem_acquire(smem);
    const int H = p.heads_v;
    const int n_pre_items = work[0] * H, n_dec_items = work[1] * H;
    const int first = static_cast<int>(blockIdx.x) < work[4] ? 0 : 1;  // 0: prefill, 1: decode

    // The next item of queue qn whose slot is in the pool (bad slots are
    // reported and skipped); every thread gets it. s < 0: the queue is empty.
    // Thread 0 claims decode rows kDecBatch at a time with one atomic and
    // resolves the batch's sequences and slots with independent loads, so a
    // row costs no chain of dependent global round trips.
    constexpr int kDecBatch = 8;
    __shared__ MixedItem dec_cache[kDecBatch];
    __shared__ int dec_n, dec_pos;
    const int n_pre = work[0];
    if (threadIdx.x == 0) dec_n = dec_pos = 0;
    auto resolve = [&](int qn, int i, int s, MixedItem& it) {
        const int slot = slots ? slots[s] : s;
        it = MixedItem{qn, s, i % H, nullptr};
        if (slot < 0 || slot >= n_slots) {
            atomicOr(&g_tc_error, 2);
            it.s = -2;  // skipped
        } else {
            it.st = pool + (static_cast<int64_t>(slot) * H + it.h) * kD * kD;
        }
    };
    auto fetch = [&](int qn) -> MixedItem {
        if (threadIdx.x == 0) {
            MixedItem it{qn, -1, 0, nullptr};
            if (qn == 0) {
                for (;;) {
                    const int i = atomicAdd(&work[2], 1);
                    if (i >= n_pre_items) break;
                    resolve(0, i, work[kWorkHeader + i / H], it);
                    if (it.s >= 0) break;
                    it.s = -1;
                }
            } else {
                for (;;) {
                    if (dec_pos == dec_n) {
                        const int i0 = atomicAdd(&work[3], kDecBatch);
                        const int n = n_dec_items - i0 < kDecBatch ? n_dec_items - i0 : kDecBatch;
                        dec_n = n > 0 ? n : 0;
                        dec_pos = 0;
                        if (dec_n == 0) break;
                        int seq[kDecBatch];
#pragma unroll
                        for (int u = 0; u < kDecBatch; ++u)
                            seq[u] = u < dec_n ? work[kWorkHeader + n_pre + (i0 + u) / H] : 0;
#pragma unroll
                        for (int u = 0; u < kDecBatch; ++u)
                            if (u < dec_n) resolve(1, i0 + u, seq[u], dec_cache[u]);
                    }
                    it = dec_cache[dec_pos++];
                    if (it.s >= 0) break;
                    it.s = -1;
                }
            }
            shared_item = it;
        }
        __syncthreads();
        const MixedItem it = shared_item;
        __syncthreads();
        return it;
    };

#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        const int qn = pass == 0 ? first : 1 - first;
        if (qn == 0) {
#pragma unroll 1
            for (MixedItem it = fetch(0); it.s >= 0; it = fetch(0)) {
                int64_t t0, t1;
                seq_span(p, it.s, t0, t1);
                prefill_item(p, &tm_q, &tm_k, &tm_v, g, beta, out, t0, t1 - t0, it.h, it.st,
                             it.st, smem, tbase);
                __syncthreads();
            }
            continue;
        }
        float* stage = reinterpret_cast<float*>(smem + kOffDecStage);
        uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffDecBar);
        fence_proxy_async();  // earlier generic use of this memory, before bulk writes
        if (threadIdx.x == 0) {
            mbar_init(bar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        auto stage_state = [&](const MixedItem& it) {  // thread 0
            mbar_expect_tx(bar, kD * kD * 4);
            bulk_load(stage, it.st, kD * kD * 4, bar);
        };
        // A row's first inputs (q, k, v, gates) load while the row before it
        // is updated, as its state does.
        auto row_in = [&](const MixedItem& it) {
            int64_t a, b;
            seq_span(p, it.s, a, b);
            return decode_in(p, q, k, v, g, beta, a, it.h);
        };
        uint32_t ph = 0;
        MixedItem cur = fetch(1);
        if (threadIdx.x == 0 && cur.s >= 0) stage_state(cur);
        DecodeIn<__nv_bfloat16> cur_in{};
        if (cur.s >= 0) cur_in = row_in(cur);
#pragma unroll 1
        while (cur.s >= 0) {
            if (!mbar_wait(bar, ph, kWaitLimitNs)) atomicOr(&g_tc_error, 1);
            ph ^= 1u;
            DecodeState st;
            decode_load_state(stage, st);
            fence_proxy_async();  // these reads, before the next bulk write
            const MixedItem next = fetch(1);  // (its barriers order the reads)
            if (threadIdx.x == 0 && next.s >= 0) stage_state(next);
            DecodeIn<__nv_bfloat16> next_in;  // read only when there is a next row
            if (next.s >= 0) next_in = row_in(next);
            int64_t t0, t1;
            seq_span(p, cur.s, t0, t1);
            decode_positions<__nv_bfloat16>(p, q, k, v, g, beta, t0, t1, cur.h, st, out, smem,
                                            cur_in);
            decode_store_state(cur.st, st);
            cur = next;
            cur_in = next_in;
        }
        __syncthreads();
        if (threadIdx.x == 0) mbar_inval(bar);
        __syncthreads();
    }
    tmem_release(tbase);
}

// ---- Sequence-parallel prefill ----------------------------------------------
// A (sequence, head) walks its chunks in order, so a pack whose longest
// sequence holds more chunks than a slot's share of the work (long sequences,
// few heads per GPU) waits on that one chain. Over positions [a, b) the
// state update is affine in the state,
//   S_b = M S_a + B,
// with M (d_k x d_k) a function of k, g and beta only, and B the state that
// the positions reach from S_a = 0. The same item run with v = 0 from S_a = I
// ends in M (a [d_k, d_v = d_k] state); run from S_a = 0 it ends in B. A long
// sequence therefore splits into P segments:
//   pass A  segment 0 from the sequence's initial state (output; its final
//           state is X_1) and, for 0 < p < P-1, the runs giving B_p and M_p
//           (no output), beside the sequences that are not split;
//   scan    X_{p+1} = M_p X_p + B_p in f32 on the CUDA cores;
//   pass B  segments 1 .. P-1 from X_p (output; the last one's final state
//           is the sequence's).
// A middle segment runs three times, so the plan weighs the longest chain
// against the extra work and splits nothing when the chain does not bound the
// call. Two segments need neither B/M runs nor a scan link: pass B's segment
// starts from the state pass A's first segment ends in.
enum : int32_t { kRunFull = 0, kRunSeg0 = 1, kRunB = 2, kRunM = 3, kRunMid = 4, kRunLast = 5 };

struct SplitDesc {
    int32_t s;     // sequence
    int32_t c0;    // first chunk of the segment
    int32_t nc;    // its chunks; -1: the whole sequence
    int32_t kind;  // kRun* | slot << 3 (the segment's index in the scratch states)
};

// Work header: [0], [1] items of pass A and pass B, [2], [3] their cursors,
// [4] split sequences, [5] segment slots used, [6] the segment length chosen
// (0: nothing split), [7] the scan's cursor.
constexpr int kSplitHeader = 16;
constexpr int kSplitCands = 16;        // segment lengths the plan tries
constexpr int kPlanCache = 4096;       // sequences whose chunk counts the plan keeps
// Costs in chunk-times (one chunk of one item with every CTA slot busy),
// fitted to B200 timings of both passes and the scan at 4 to 32 value heads.
constexpr float kItemCost = 0.5f;       // per item: state in and out, setup
constexpr float kAloneFactor = 0.75f;   // a chunk when at most one CTA per SM is busy
constexpr float kScanStepCost = 1.1f;   // one link of the longest scan chain
constexpr float kScanLaunchCost = 1.0f;
constexpr int kScanBlocks = 8;          // column blocks of a (sequence, head) scan

// A pass of `n` items (`work` chunk-times in all, the longest `longest`) on
// `slots` CTA slots, as the longest-first list schedule runs it: one wave
// when the items fit the slots, else the longest item or the average load
// plus half an average item, whichever is more (a replay of that schedule on
// the ragged pack's passes at 2 to 32 value heads agrees within a few
// chunk-times).
__device__ __forceinline__ float pass_time(float n, float work, float longest, float slots) {
    if (n <= 0.f) return 0.f;
    if (n <= slots) return longest * (n <= 0.5f * slots ? kAloneFactor : 1.f);
    return fmaxf(work / slots + 0.5f * work / n, longest);
}

__device__ __forceinline__ int seg_begin(int c, int parts, int i) {
    return static_cast<int>(static_cast<int64_t>(i) * c / parts);
}

// Exclusive prefix sum of a[0 .. 1023] in place, by a CTA of 1024 threads;
// returns the total to every thread. `ws` holds 33 ints.
__device__ int exclusive_scan_1024(int* a, int* ws) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int x = a[tid];
    int inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) ws[w] = inc;
    __syncthreads();
    if (w == 0) {
        const int t = ws[lane];
        int it = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, it, o);
            if (lane >= o) it += y;
        }
        ws[lane] = it - t;
        if (lane == 31) ws[32] = it;
    }
    __syncthreads();
    a[tid] = inc - x + ws[w];
    const int total = ws[32];
    __syncthreads();
    return total;
}

// One CTA of 1024 threads (one per length bucket). Candidate segment lengths l_min * 1.15^i (or
// `forced` alone) are scored as
//   max(work_A / slots, longest item of A) + max(work_B / slots, longest of B)
// in chunk-times, against max(work / slots, longest sequence) unsplit; the
// best one is used if it beats not splitting (`forced` is used whenever it
// splits anything). Items of each pass are listed longest first.
__global__ void __launch_bounds__(1024)
plan_split(const Problem p, int32_t* work, SplitDesc* da, SplitDesc* db, int4* splits,
           int slots, int l_min, int forced, int seg_cap) {
    // Per candidate: work and longest item of each pass, segments, split
    // sequences, scan steps (total and longest chain); [kSplitCands]: unsplit.
    __shared__ float est_work_a[kSplitCands + 1], est_max_a[kSplitCands + 1],
        est_work_b[kSplitCands], est_max_b[kSplitCands];
    __shared__ int est_items_a[kSplitCands + 1], est_items_b[kSplitCands];
    __shared__ int est_segs[kSplitCands], est_split[kSplitCands], est_chain[kSplitCands];
    __shared__ int hist[3][kPlanBuckets];  // pass A items, pass B items, split sequences
    __shared__ int chosen, n_split, n_slot;
    __shared__ int warp_sums[33];
    int n_a, n_b;
    const int n = p.n_seqs, H = p.heads_v, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int n_cand = forced > 0 ? 1 : kSplitCands;
    auto cand = [&](int i) {
        return forced > 0 ? forced : static_cast<int>(l_min * __powf(1.15f, static_cast<float>(i)));
    };
    // Chunk counts, read from the offsets once and kept for the first
    // kPlanCache sequences (the three passes below read them again).
    __shared__ int ccache[kPlanCache];
    auto chunks_global = [&](int s) {
        int64_t a, b;
        seq_span(p, s, a, b);
        return static_cast<int>((b - a + kC - 1) / kC);
    };
    auto chunks_of = [&](int s) { return s < kPlanCache ? ccache[s] : chunks_global(s); };
    auto bucket = [&](int c) {  // descending chunk count
        return kPlanBuckets - 1 - (c < kPlanBuckets - 1 ? c : kPlanBuckets - 1);
    };
    for (int i = tid; i < kPlanBuckets; i += blockDim.x) hist[0][i] = hist[1][i] = hist[2][i] = 0;
    for (int i = tid; i < n && i < kPlanCache; i += blockDim.x) ccache[i] = chunks_global(i);
    if (tid == 0) n_split = n_slot = 0;
    __syncthreads();
    // Warp i scores candidate i (warp kSplitCands: no split), lanes over the
    // sequences, then one warp reduction.
    if (warp <= kSplitCands && (warp < n_cand || warp == kSplitCands)) {
        const int L = warp < kSplitCands ? cand(warp) : 0;
        float wa = 0.f, ma = 0.f, wb = 0.f, mb = 0.f;
        int na = 0, nb = 0, segs = 0, nsp = 0, chain = 0;
        for (int s = lane; s < n; s += 32) {
            const int c = chunks_of(s);
            const int parts = L > 0 ? (c + L - 1) / L : 1;
            if (parts < 2) {
                wa += c + kItemCost;
                ma = fmaxf(ma, c + kItemCost);
                na += 1;
                continue;
            }
            // Segment sizes are floor(c / parts) or one more; the first is
            // the floor.
            const float first = static_cast<float>(c / parts);
            const float last = static_cast<float>(c - seg_begin(c, parts, parts - 1));
            const float big = static_cast<float>((c + parts - 1) / parts);
            const float mid = static_cast<float>(c) - first - last;
            wa += first + kItemCost + 2.f * (mid + (parts - 2) * kItemCost);
            wb += static_cast<float>(c) - first + (parts - 1) * kItemCost;
            ma = fmaxf(ma, big + kItemCost);
            mb = fmaxf(mb, big + kItemCost);
            na += 1 + 2 * (parts - 2);
            nb += parts - 1;
            segs += parts;
            nsp += 1;
            chain = max(chain, parts - 2);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            wa += __shfl_xor_sync(0xffffffffu, wa, o);
            wb += __shfl_xor_sync(0xffffffffu, wb, o);
            na += __shfl_xor_sync(0xffffffffu, na, o);
            nb += __shfl_xor_sync(0xffffffffu, nb, o);
            ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
            mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            segs += __shfl_xor_sync(0xffffffffu, segs, o);
            nsp += __shfl_xor_sync(0xffffffffu, nsp, o);
            chain = max(chain, __shfl_xor_sync(0xffffffffu, chain, o));
        }
        if (lane == 0) {
            est_work_a[warp] = wa;
            est_max_a[warp] = ma;
            est_items_a[warp] = na;
            if (warp < kSplitCands) {
                est_work_b[warp] = wb;
                est_max_b[warp] = mb;
                est_items_b[warp] = nb;
                est_segs[warp] = segs;
                est_split[warp] = nsp;
                est_chain[warp] = chain;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        const float fh = static_cast<float>(H), fs = static_cast<float>(slots);
        auto pass = [&](int items, float work, float longest) {
            return pass_time(items * fh, work * fh, longest, fs);
        };
        const int u = kSplitCands;
        float best = forced > 0 ? INFINITY : pass(est_items_a[u], est_work_a[u], est_max_a[u]);
        int best_l = 0;
        for (int i = 0; i < n_cand; ++i) {
            if (est_split[i] == 0 || est_segs[i] > seg_cap) continue;
            const float est = pass(est_items_a[i], est_work_a[i], est_max_a[i]) +
                              pass(est_items_b[i], est_work_b[i], est_max_b[i]) +
                              kScanLaunchCost + kScanStepCost * est_chain[i];
            if (est < best) {
                best = est;
                best_l = cand(i);
            }
        }
        chosen = best_l;
    }
    __syncthreads();
    const int L = chosen;
    auto parts_of = [&](int c) { return L > 0 ? (c + L - 1) / L : 1; };
    for (int s = tid; s < n; s += blockDim.x) {  // count the items by length
        const int c = chunks_of(s), parts = parts_of(c);
        if (parts < 2) {
            atomicAdd(&hist[0][bucket(c)], 1);
            continue;
        }
        atomicAdd(&hist[2][bucket(c)], 1);
        for (int j = 0; j < parts; ++j) {
            const int cs = seg_begin(c, parts, j + 1) - seg_begin(c, parts, j);
            if (j == 0) {
                atomicAdd(&hist[0][bucket(cs)], 1);
            } else {
                atomicAdd(&hist[1][bucket(cs)], 1);
                if (j < parts - 1) atomicAdd(&hist[0][bucket(cs)], 2);
            }
        }
    }
    __syncthreads();
    n_a = exclusive_scan_1024(hist[0], warp_sums);  // bucket counts -> cursors
    n_b = exclusive_scan_1024(hist[1], warp_sums);
    exclusive_scan_1024(hist[2], warp_sums);  // split sequences, longest first
    for (int s = tid; s < n; s += blockDim.x) {  // place them
        const int c = chunks_of(s), parts = parts_of(c);
        if (parts < 2) {
            da[atomicAdd(&hist[0][bucket(c)], 1)] = SplitDesc{s, 0, -1, kRunFull};
            continue;
        }
        const int j = atomicAdd(&hist[2][bucket(c)], 1);
        atomicAdd(&n_split, 1);
        const int base = atomicAdd(&n_slot, parts);
        splits[j] = make_int4(base, parts, s, 0);
        for (int i = 0; i < parts; ++i) {
            const int b0 = seg_begin(c, parts, i), cs = seg_begin(c, parts, i + 1) - b0;
            const int slot = (base + i) << 3;
            if (i == 0) {
                da[atomicAdd(&hist[0][bucket(cs)], 1)] = SplitDesc{s, b0, cs, kRunSeg0 | slot};
                continue;
            }
            db[atomicAdd(&hist[1][bucket(cs)], 1)] =
                SplitDesc{s, b0, cs, (i == parts - 1 ? kRunLast : kRunMid) | slot};
            if (i < parts - 1) {
                const int at = atomicAdd(&hist[0][bucket(cs)], 2);
                da[at] = SplitDesc{s, b0, cs, kRunB | slot};
                da[at + 1] = SplitDesc{s, b0, cs, kRunM | slot};
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        work[0] = n_a;
        work[1] = n_b;
        work[2] = 0;
        work[3] = 0;
        work[4] = n_split;
        work[5] = n_slot;
        work[6] = L;
        work[7] = 0;
    }
}

// The three scratch states of a segment slot: X (the state at the segment's
// start), B and M, each [slot][head][d_k][d_v] f32.
__device__ __forceinline__ float* split_state(float* scratch, int seg_cap, int heads, int which,
                                              int slot, int h) {
    return scratch +
           ((static_cast<int64_t>(which) * seg_cap + slot) * heads + h) * static_cast<int64_t>(kD * kD);
}

// Pass A (`which` 0) or pass B (1): CTAs pull (item, value head) pairs, the
// value heads of one item next to each other so the two heads of a key head
// share its tiles in L2. Each CTA holds its TMEM columns for all its items.
__global__ void __launch_bounds__(kThreads, 2)
split_pass(const Problem p, const __grid_constant__ CUtensorMap tm_q,
           const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
           const float* __restrict__ g, const float* __restrict__ beta, const float* state_in,
           __nv_bfloat16* __restrict__ out, float* state_out, int32_t* work,
           const SplitDesc* __restrict__ desc, int which, float* scratch, int seg_cap) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = aligned_smem(smem_raw);
    __shared__ int item;
    const int H = p.heads_v;
    const int n_items = work[which] * H;
    // With fewer items than CTAs, the first CTAs (one per SM before any SM
    // gets a second) run them and the rest leave.
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    const uint32_t tbase = tmem_acquire(smem);
#pragma unroll 1
    for (;;) {
        if (threadIdx.x == 0) item = atomicAdd(&work[2 + which], 1);
        __syncthreads();
        const int i = item;
        __syncthreads();
        if (i >= n_items) break;
        const SplitDesc d = desc[i / H];
        const int h = i % H;
        int64_t a, b;
        seq_span(p, d.s, a, b);
        int64_t t0 = a, len = b - a;
        if (d.nc >= 0) {
            t0 = a + static_cast<int64_t>(d.c0) * kC;
            const int64_t e = t0 + static_cast<int64_t>(d.nc) * kC;
            len = (e < b ? e : b) - t0;
        }
        const int kind = d.kind & 7, slot = d.kind >> 3;
        const int64_t hs = (static_cast<int64_t>(d.s) * H + h) * kD * kD;
        const float* in = nullptr;
        float* fin = nullptr;
        switch (kind) {
            case kRunFull:
                in = state_in ? state_in + hs : nullptr;
                fin = state_out + hs;
                break;
            case kRunSeg0:
                in = state_in ? state_in + hs : nullptr;
                fin = split_state(scratch, seg_cap, H, 0, slot + 1, h);
                break;
            case kRunB:
                fin = split_state(scratch, seg_cap, H, 1, slot, h);
                break;
            case kRunM:
                fin = split_state(scratch, seg_cap, H, 2, slot, h);
                break;
            case kRunMid:
                in = split_state(scratch, seg_cap, H, 0, slot, h);
                break;
            default:  // kRunLast
                in = split_state(scratch, seg_cap, H, 0, slot, h);
                fin = state_out + hs;
                break;
        }
        if (kind == kRunB)
            prefill_item<kItemNoOut>(p, &tm_q, &tm_k, &tm_v, g, beta, out, t0, len, h, in, fin,
                                     smem, tbase);
        else if (kind == kRunM)
            prefill_item<kItemIdentity | kItemZeroV | kItemNoOut>(
                p, &tm_q, &tm_k, &tm_v, g, beta, out, t0, len, h, in, fin, smem, tbase);
        else
            prefill_item(p, &tm_q, &tm_k, &tm_v, g, beta, out, t0, len, h, in, fin, smem, tbase);
        __syncthreads();
    }
    tmem_release(tbase);
}

// X_{p+1} = M_p X_p + B_p for p = 1 .. P-2 of every split sequence and value
// head, a block of kScanCols state columns per item (the columns of S evolve
// independently); CTAs pull items, the longest chains first. M_p is staged
// whole in shared memory by cp.async (every copy in flight at once). The
// product runs on the tensor cores as tf32 m16n8k8 mma.sync in three parts,
// hi.hi + hi.lo + lo.hi with x = hi + lo split to tf32 (the split keeps about
// f32 accuracy): warp w computes rows 16 w .. 16 w + 15 of the block's 16
// columns. Rows of M_p are padded to 132 floats and of the state block to 24,
// so each fragment load meets 32 distinct banks. Eight 16-column blocks per
// (sequence, head) measured faster than four of 32 (the chain of links is the
// longest item; its work per link halves, its load of M_p does not) and than
// sixteen of 8.
constexpr int kScanCols = kD / kScanBlocks;
constexpr int kScanPad = kD + 4;
constexpr int kScanSPad = kScanCols + 8;
constexpr uint32_t kScanSmem = (kD * kScanPad + kD * kScanSPad) * 4;
constexpr int kScanNT = kScanCols / 8;  // n-tiles of 8 columns per warp
static_assert(kScanCols % 8 == 0, "whole n-tiles");

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    const float r = x - __uint_as_float(hi);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__global__ void __launch_bounds__(256, 2)
split_scan(int32_t* work, const int4* splits, float* scratch, int seg_cap, int H) {
    extern __shared__ float ssm[];
    float* Ms = ssm;
    float* Ss = ssm + kD * kScanPad;
    __shared__ int item;
    const int n_items = work[4] * H * kScanBlocks;
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    const int tid = threadIdx.x, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
    const int rw = 16 * (tid >> 5);  // this warp's first row
    auto copy16 = [](float* dst, const float* src) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                     : "memory");
    };
#pragma unroll 1
    for (;;) {
        if (tid == 0) item = atomicAdd(&work[7], 1);
        __syncthreads();
        const int it = item;
        __syncthreads();
        if (it >= n_items) break;
        const int cb = it % kScanBlocks, jh = it / kScanBlocks;
        const int h = jh % H;
        const int4 sp = splits[jh / H];
        const int base = sp.x, parts = sp.y;
        if (parts < 3) continue;  // two segments: no link (every thread sees the same item)
        const int col0 = cb * kScanCols;
        {
            const float* x1 = split_state(scratch, seg_cap, H, 0, base + 1, h);
            for (int e = tid; e < kD * kScanCols / 4; e += blockDim.x) {
                const int row = e / (kScanCols / 4), c4 = e % (kScanCols / 4);
                copy16(Ss + row * kScanSPad + 4 * c4, x1 + row * kD + col0 + 4 * c4);
            }
        }
#pragma unroll 1
        for (int j = 1; j + 1 < parts; ++j) {
            const float* m = split_state(scratch, seg_cap, H, 2, base + j, h);
#pragma unroll
            for (int u = 0; u < kD * kD / 4 / 256; ++u) {
                const int e = tid + 256 * u;
                const int row = e / (kD / 4), c = 4 * (e % (kD / 4));
                copy16(Ms + row * kScanPad + c, m + 4 * e);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            // C starts as B_p: fragment (row rw + gq (+8), column 8 nt + 2 tq (+1)).
            const float* bp = split_state(scratch, seg_cap, H, 1, base + j, h) + col0;
            float c[kScanNT][4];
#pragma unroll
            for (int nt = 0; nt < kScanNT; ++nt) {
                const float2 u = *reinterpret_cast<const float2*>(bp + (rw + gq) * kD + 8 * nt + 2 * tq);
                const float2 v = *reinterpret_cast<const float2*>(bp + (rw + gq + 8) * kD + 8 * nt + 2 * tq);
                c[nt][0] = u.x, c[nt][1] = u.y, c[nt][2] = v.x, c[nt][3] = v.y;
            }
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            __syncthreads();
#pragma unroll 2
            for (int ks = 0; ks < kD / 8; ++ks) {
                const float* ma = Ms + (rw + gq) * kScanPad + 8 * ks + tq;
                uint32_t ah[4], al[4];
                tf32_split(ma[0], ah[0], al[0]);
                tf32_split(ma[8 * kScanPad], ah[1], al[1]);
                tf32_split(ma[4], ah[2], al[2]);
                tf32_split(ma[8 * kScanPad + 4], ah[3], al[3]);
                const float* sb = Ss + (8 * ks + tq) * kScanSPad + gq;
#pragma unroll
                for (int nt = 0; nt < kScanNT; ++nt) {
                    uint32_t bh0, bl0, bh1, bl1;
                    tf32_split(sb[8 * nt], bh0, bl0);
                    tf32_split(sb[4 * kScanSPad + 8 * nt], bh1, bl1);
                    mma_tf32(c[nt], ah, bh0, bh1);
                    mma_tf32(c[nt], ah, bl0, bl1);
                    mma_tf32(c[nt], al, bh0, bh1);
                }
            }
            __syncthreads();  // every read of Ss and Ms is done
            float* xn = split_state(scratch, seg_cap, H, 0, base + j + 1, h) + col0;
#pragma unroll
            for (int nt = 0; nt < kScanNT; ++nt) {
                const int cc = 8 * nt + 2 * tq;
                const float2 top = make_float2(c[nt][0], c[nt][1]);
                const float2 bot = make_float2(c[nt][2], c[nt][3]);
                *reinterpret_cast<float2*>(Ss + (rw + gq) * kScanSPad + cc) = top;
                *reinterpret_cast<float2*>(Ss + (rw + gq + 8) * kScanSPad + cc) = bot;
                *reinterpret_cast<float2*>(xn + (rw + gq) * kD + cc) = top;
                *reinterpret_cast<float2*>(xn + (rw + gq + 8) * kD + cc) = bot;
            }
            __syncthreads();
        }
        __syncthreads();
    }
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

// A self-test of the bounded waits: one thread waits, at most `limit_ns`, for
// an mbarrier phase that nothing completes, with the same wait the kernels
// use; when the wait gives up it records the failure exactly as they do.
__global__ void selftest_wait(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (!mbar_wait(&bar, 0, limit_ns)) atomicOr(&g_tc_error, 1);
    mbar_inval(&bar);
}

cudaError_t launch_selftest_wait(uint64_t limit_ns, cudaStream_t stream) {
    selftest_wait<<<1, 32, 0, stream>>>(limit_ns);
    return cudaGetLastError();
}

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

static cudaError_t make_maps(const Problem& p, const void* q, const void* k, const void* v,
                             const void* out, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv) {
    const uintptr_t align = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                            reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
    if (align & 15) return cudaErrorMisalignedAddress;
    const int64_t tokens = p.cu_seqlens ? p.seq_len : static_cast<int64_t>(p.n_seqs) * p.seq_len;
    if (tokens >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
    if (!make_map(mq, q, tokens, p.heads_qk) || !make_map(mk, k, tokens, p.heads_qk) ||
        !make_map(mv, v, tokens, p.heads_v))
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

template <typename K>
static cudaError_t allow_smem(K* kernel) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmemBytes));
}

cudaError_t launch_chunked_tc(const Problem& p, const void* q, const void* k, const void* v,
                              const float* g, const float* beta, const float* state_in, void* out,
                              float* state_out, cudaStream_t stream) {
    CUtensorMap mq, mk, mv;
    cudaError_t e = make_maps(p, q, k, v, out, &mq, &mk, &mv);
    if (e != cudaSuccess) return e;
    if ((e = allow_smem(chunked_tc)) != cudaSuccess) return e;
    chunked_tc<<<dim3(p.heads_v, p.n_seqs), kThreads, kSmemBytes, stream>>>(
        p, mq, mk, mv, g, beta, state_in, static_cast<__nv_bfloat16*>(out), state_out);
    return cudaGetLastError();
}

size_t mixed_workspace_bytes(int n_seqs) {
    return (static_cast<size_t>(n_seqs) + kWorkHeader) * sizeof(int32_t);
}

static int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    return n;
}

cudaError_t launch_mixed_tc(const Problem& p, const void* q, const void* k, const void* v,
                            const float* g, const float* beta, float* pool, const int32_t* slots,
                            int32_t n_slots, void* out, int32_t* work, cudaStream_t stream) {
    CUtensorMap mq, mk, mv;
    cudaError_t e = make_maps(p, q, k, v, out, &mq, &mk, &mv);
    if (e != cudaSuccess) return e;
    if ((e = allow_smem(mixed_tc)) != cudaSuccess) return e;
    const int64_t items = static_cast<int64_t>(p.n_seqs) * p.heads_v;
    const int grid = static_cast<int>(items < 2 * sm_count() ? items : 2 * sm_count());
    plan_mixed<<<1, 1024, 0, stream>>>(p, work, grid);
    mixed_tc<<<grid, kThreads, kSmemBytes, stream>>>(
        p, mq, mk, mv, static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
        static_cast<const __nv_bfloat16*>(v), g, beta, pool, slots, n_slots,
        static_cast<__nv_bfloat16*>(out), work);
    return cudaGetLastError();
}

// ---- gdr_mixed without a caller workspace ----------------------------------
// The work list of gdr_mixed_noalloc lives in this fixed device array instead
// of caller-provided memory: an 8-word header plus one entry per sequence, for at
// most kMixedNoAllocMaxSeqs sequences (64 KiB). Every GPU that loads the
// library holds one copy until the process exits. All calls on a device share
// it and it keeps the previous call's contents; the planning kernel rewrites
// every entry a call reads and zeroes the two queue cursors the launch counts
// up from, so nothing stale is read, but calls whose work
// overlaps on the GPU (different streams, no ordering between them) race on
// it.
constexpr int kMixedNoAllocMaxSeqs = GDR_MIXED_NOALLOC_MAX_SEQS;
static __device__ __align__(256) int32_t g_mixed_scratch[kWorkHeader + kMixedNoAllocMaxSeqs];

// The device address of g_mixed_scratch on the current device, looked up once
// per device (host code cannot use the symbol itself as a device pointer).
static cudaError_t mixed_scratch_ptr(int32_t** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static int32_t* ptrs[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_mixed_scratch);
        if (e != cudaSuccess) return e;
        ptrs[dev] = static_cast<int32_t*>(ptr);
    }
    *out = ptrs[dev];
    return cudaSuccess;
}

int mixed_noalloc_max_seqs() { return kMixedNoAllocMaxSeqs; }

cudaError_t launch_mixed_tc_noalloc(const Problem& p, const void* q, const void* k,
                                    const void* v, const float* g, const float* beta,
                                    float* pool, const int32_t* slots, int32_t n_slots,
                                    void* out, cudaStream_t stream) {
    int32_t* work = nullptr;
    cudaError_t e = mixed_scratch_ptr(&work);
    if (e != cudaSuccess) return e;
    return launch_mixed_tc(p, q, k, v, g, beta, pool, slots, n_slots, out, work, stream);
}

}  // namespace gdr

// ---- Sequence-parallel launch (GDR_ALGO_TENSOR_SPLIT) ----------------------
namespace gdr {
namespace {

constexpr int kMinSegChunks = 4;
constexpr size_t kSplitStateBudget = size_t{2} << 30;  // scratch states, bytes

}  // namespace

// The stream-ordered pool the library's scratch comes from (split calls,
// host-buffer calls): one per device, owned by the library. Its release
// threshold keeps freed memory reserved so repeated calls reuse it;
// gdr_release_scratch gives it back. With create false, a device without a
// pool yet gets a null pool.
cudaError_t library_pool(cudaMemPool_t* pool, bool create) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static cudaMemPool_t pools[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (pools[dev] == nullptr && create) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t made = nullptr;
        if ((e = cudaMemPoolCreate(&made, &props)) != cudaSuccess) return e;
        uint64_t keep = UINT64_MAX;
        if ((e = cudaMemPoolSetAttribute(made, cudaMemPoolAttrReleaseThreshold, &keep)) !=
            cudaSuccess) {
            cudaMemPoolDestroy(made);  // a later call tries again from scratch
            return e;
        }
        pools[dev] = made;
    }
    *pool = pools[dev];
    return cudaSuccess;
}

namespace {

// Host-side sizes of a split call: the smallest segment length the plan may
// pick and the segment slots that bounds.
struct SplitShape {
    int slots;      // CTA slots (two per SM)
    int l_min;      // chunks
    int max_chunks; // of the longest possible sequence
    int seg_cap;    // segment slots
};

SplitShape split_shape(const Problem& p, int forced) {
    SplitShape sh;
    sh.slots = 2 * sm_count();
    const int64_t tokens = p.cu_seqlens ? p.seq_len : static_cast<int64_t>(p.n_seqs) * p.seq_len;
    const int64_t longest = p.cu_seqlens ? tokens : p.seq_len;
    sh.max_chunks = static_cast<int>((longest + kC - 1) / kC);
    const int64_t chunks = p.cu_seqlens ? (tokens + kC - 1) / kC + p.n_seqs
                                        : static_cast<int64_t>(p.n_seqs) * sh.max_chunks;
    const double avg = static_cast<double>(chunks) * p.heads_v / sh.slots;
    sh.l_min = forced > 0 ? forced : std::max(kMinSegChunks, static_cast<int>(0.35 * avg));
    // A split sequence has P = ceil(c / L) >= 2 segments (c > L), so P < 2 c / L.
    const int64_t cap = static_cast<int64_t>(2.1 * static_cast<double>(chunks) / sh.l_min) + 2;
    const int64_t budget = static_cast<int64_t>(
        kSplitStateBudget / (3 * static_cast<size_t>(p.heads_v) * kD * kD * sizeof(float)));
    sh.seg_cap = static_cast<int>(std::max<int64_t>(3, std::min(cap, budget)));
    return sh;
}

}  // namespace

// GDR_ALGO_AUTO's choice: split when some sequence could be longer than two
// of the shortest segments worth running.
bool split_may_help(const Problem& p) {
    const SplitShape sh = split_shape(p, 0);
    return sh.max_chunks > 2 * sh.l_min;
}

cudaError_t launch_chunked_split(const Problem& p, const void* q, const void* k, const void* v,
                                 const float* g, const float* beta, const float* state_in,
                                 void* out, float* state_out, int forced, cudaStream_t stream) {
    CUtensorMap mq, mk, mv;
    cudaError_t e = make_maps(p, q, k, v, out, &mq, &mk, &mv);
    if (e != cudaSuccess) return e;
    if ((e = allow_smem(split_pass)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(split_scan, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kScanSmem))) != cudaSuccess)
        return e;
    const SplitShape sh = split_shape(p, forced);
    const size_t cap_a = static_cast<size_t>(p.n_seqs) + 2 * static_cast<size_t>(sh.seg_cap);
    const size_t cap_b = static_cast<size_t>(sh.seg_cap);
    const size_t cap_s = static_cast<size_t>(sh.seg_cap) / 2 + 1;  // >= 2 segments each
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    const size_t off_a = up(kSplitHeader * sizeof(int32_t));
    const size_t off_b = off_a + up(cap_a * sizeof(SplitDesc));
    const size_t off_s = off_b + up(cap_b * sizeof(SplitDesc));
    const size_t off_x = off_s + up(cap_s * sizeof(int4));
    const size_t bytes =
        off_x + 3 * static_cast<size_t>(sh.seg_cap) * p.heads_v * kD * kD * sizeof(float);
    cudaMemPool_t pool;
    if ((e = library_pool(&pool, true)) != cudaSuccess) return e;
    void* mem = nullptr;
    if ((e = cudaMallocFromPoolAsync(&mem, bytes, pool, stream)) != cudaSuccess) return e;
    uint8_t* base = static_cast<uint8_t*>(mem);
    int32_t* work = reinterpret_cast<int32_t*>(base);
    SplitDesc* da = reinterpret_cast<SplitDesc*>(base + off_a);
    SplitDesc* db = reinterpret_cast<SplitDesc*>(base + off_b);
    int4* splits = reinterpret_cast<int4*>(base + off_s);
    float* scratch = reinterpret_cast<float*>(base + off_x);
    auto* o = static_cast<__nv_bfloat16*>(out);
    plan_split<<<1, 1024, 0, stream>>>(p, work, da, db, splits, sh.slots, sh.l_min, forced,
                                       sh.seg_cap);
    split_pass<<<sh.slots, kThreads, kSmemBytes, stream>>>(p, mq, mk, mv, g, beta, state_in, o,
                                                          state_out, work, da, 0, scratch,
                                                          sh.seg_cap);
    split_scan<<<2 * sm_count(), 256, kScanSmem, stream>>>(work, splits, scratch, sh.seg_cap,
                                                          p.heads_v);
    split_pass<<<sh.slots, kThreads, kSmemBytes, stream>>>(p, mq, mk, mv, g, beta, state_in, o,
                                                          state_out, work, db, 1, scratch,
                                                          sh.seg_cap);
    e = cudaGetLastError();
    const cudaError_t f = cudaFreeAsync(mem, stream);
    return e != cudaSuccess ? e : f;
}

}  // namespace gdr
