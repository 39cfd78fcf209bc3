// CPU oracle for the gated delta rule -- TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain C++17, the arithmetic of bunsen's
// `GatedDeltaRule` (crates/public/bunsen/src/ops/transformers/linear_attention/
// delta_rule.rs) so that the CUDA kernels of this repository can be checked
// against it. Only the tests, the smoke check and the CPU-baseline leg of the
// benchmark load it; the product library never links or calls it.
//
// Three forms, each on a packed ragged batch (`cu_seqlens`; a dense [B, T]
// batch is the pack with cu_seqlens = 0, T, 2T, ...):
//   * gdr_oracle_scalar_f64  -- the test-only scalar rule in f64
//                               (delta_rule.rs:399-445);
//   * gdr_oracle_recurrent   -- `GatedDeltaRule::recurrent` in f32
//                               (delta_rule.rs:182-209);
//   * gdr_oracle_chunked     -- `GatedDeltaRule::chunked` in f32
//                               (delta_rule.rs:223-310, unit_lower_inverse
//                               :337-351), same operation order: prepare,
//                               pad, cumsum, pairwise decay, Gram products,
//                               row forward substitution, chunk loop.
// `prepare` (delta_rule.rs:127-165): q and k are L2-normalised as
// x / sqrt(sum x^2 + eps) when eps >= 0, and q is then divided by sqrt(d_k).
// Grouped heads follow `repeat_interleave` (ops/repeat.rs:51-66) as the
// GatedDeltaNet call site applies it (gated_delta_net.rs:404-419): value head
// h reads key/query head h / (H_v / H_qk).
//
// Work is spread over (sequence, head) pairs with OpenMP; each pair is
// computed by one thread in the order given above, so results do not depend
// on the thread count.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <omp.h>

extern "C" {

// The batch a call works on. All tensors are row-major:
//   q, k  [T_total, H_qk, d_k]     v, out [T_total, H_v, d_v]
//   g, beta [T_total, H_v]          state_in/state_out [n_seqs, H_v, d_k, d_v]
// state_in may be null (zeros). cu_seqlens has n_seqs + 1 entries.
struct gdr_oracle_batch {
    int32_t n_seqs;
    const int32_t* cu_seqlens;
    int32_t heads_qk;
    int32_t heads_v;
    int32_t d_k;
    int32_t d_v;
    int32_t chunk_size;  // chunked form only
    double l2norm_eps;   // < 0: no normalisation (qk_l2norm_eps = None)
    int32_t threads;     // <= 0: all of OpenMP's threads
};

}  // extern "C"

namespace {

template <typename F>
struct View {
    const gdr_oracle_batch& b;
    int64_t row_qk(int64_t t, int h) const {
        const int group = b.heads_v / b.heads_qk;
        return (t * b.heads_qk + h / group) * b.d_k;
    }
    int64_t row_v(int64_t t, int h) const { return (t * b.heads_v + h) * b.d_v; }
    int64_t gate(int64_t t, int h) const { return t * b.heads_v + h; }
    int64_t state(int s, int h) const {
        return (static_cast<int64_t>(s) * b.heads_v + h) * b.d_k * b.d_v;
    }
};

bool valid(const gdr_oracle_batch* b) {
    if (!b || b->n_seqs < 0 || !b->cu_seqlens || b->heads_qk <= 0 || b->heads_v <= 0 ||
        b->d_k <= 0 || b->d_v <= 0 || b->heads_v % b->heads_qk != 0)
        return false;
    for (int s = 0; s < b->n_seqs; ++s)
        if (b->cu_seqlens[s + 1] < b->cu_seqlens[s]) return false;
    return b->cu_seqlens[0] == 0;
}

// delta_rule.rs:112-123 and :153-154: x / sqrt(sum x^2 + eps), then for
// queries a division by sqrt(d_k).
template <typename F>
void prepare_vec(const F* x, int d, double eps, bool query, F* y) {
    if (eps >= 0) {
        F ss = 0;
        for (int i = 0; i < d; ++i) ss += x[i] * x[i];
        const F norm = std::sqrt(ss + static_cast<F>(eps));
        for (int i = 0; i < d; ++i) y[i] = x[i] / norm;
    } else {
        for (int i = 0; i < d; ++i) y[i] = x[i];
    }
    if (query) {
        const F root = std::sqrt(static_cast<F>(d));
        for (int i = 0; i < d; ++i) y[i] = y[i] / root;
    }
}

template <typename F>
int for_pairs(const gdr_oracle_batch* b, F body) {
    const int pairs = b->n_seqs * b->heads_v;
    const int threads = b->threads > 0 ? b->threads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int p = 0; p < pairs; ++p) body(p / b->heads_v, p % b->heads_v);
    return 0;
}

// ---- the scalar rule, f64 (delta_rule.rs:399-445) ------------------------
int scalar_f64(const gdr_oracle_batch* b, const double* q, const double* k, const double* v,
               const double* g, const double* beta, const double* state_in, double* out,
               double* state_out) {
    View<double> at{*b};
    const int dk = b->d_k, dv = b->d_v;
    return for_pairs(b, [&](int s, int h) {
        double* st = state_out + at.state(s, h);
        if (state_in)
            std::memmove(st, state_in + at.state(s, h), sizeof(double) * dk * dv);
        else
            std::fill(st, st + dk * dv, 0.0);
        std::vector<double> qt(dk), kt(dk);
        for (int t = b->cu_seqlens[s]; t < b->cu_seqlens[s + 1]; ++t) {
            prepare_vec(q + at.row_qk(t, h), dk, b->l2norm_eps, true, qt.data());
            prepare_vec(k + at.row_qk(t, h), dk, b->l2norm_eps, false, kt.data());
            const double* vt = v + at.row_v(t, h);
            const double decay = std::exp(g[at.gate(t, h)]);
            for (int i = 0; i < dk * dv; ++i) st[i] *= decay;
            for (int j = 0; j < dv; ++j) {
                double read = 0;
                for (int i = 0; i < dk; ++i) read += st[i * dv + j] * kt[i];
                const double delta = (vt[j] - read) * beta[at.gate(t, h)];
                for (int i = 0; i < dk; ++i) st[i * dv + j] += kt[i] * delta;
            }
            double* o = out + at.row_v(t, h);
            for (int j = 0; j < dv; ++j) {
                double acc = 0;
                for (int i = 0; i < dk; ++i) acc += st[i * dv + j] * qt[i];
                o[j] = acc;
            }
        }
    });
}

// ---- GatedDeltaRule::recurrent, f32 (delta_rule.rs:182-209) ---------------
int recurrent_f32(const gdr_oracle_batch* b, const float* q, const float* k, const float* v,
                  const float* g, const float* beta, const float* state_in, float* out,
                  float* state_out) {
    View<float> at{*b};
    const int dk = b->d_k, dv = b->d_v;
    return for_pairs(b, [&](int s, int h) {
        float* st = state_out + at.state(s, h);
        if (state_in)
            std::memmove(st, state_in + at.state(s, h), sizeof(float) * dk * dv);
        else
            std::fill(st, st + dk * dv, 0.0f);
        std::vector<float> qt(dk), kt(dk), read(dv), delta(dv);
        for (int t = b->cu_seqlens[s]; t < b->cu_seqlens[s + 1]; ++t) {
            prepare_vec(q + at.row_qk(t, h), dk, b->l2norm_eps, true, qt.data());
            prepare_vec(k + at.row_qk(t, h), dk, b->l2norm_eps, false, kt.data());
            const float* vt = v + at.row_v(t, h);
            const float decay = std::exp(g[at.gate(t, h)]);  // :193
            const float bt = beta[at.gate(t, h)];
            for (int i = 0; i < dk * dv; ++i) st[i] *= decay;  // :200
            // :202 read = k_t S  ([1, d_k] x [d_k, d_v])
            std::fill(read.begin(), read.end(), 0.0f);
            for (int i = 0; i < dk; ++i)
                for (int j = 0; j < dv; ++j) read[j] += kt[i] * st[i * dv + j];
            for (int j = 0; j < dv; ++j) delta[j] = (vt[j] - read[j]) * bt;  // :203
            for (int i = 0; i < dk; ++i)                                      // :204
                for (int j = 0; j < dv; ++j) st[i * dv + j] += kt[i] * delta[j];
            float* o = out + at.row_v(t, h);  // :205 o = q_t S
            for (int j = 0; j < dv; ++j) o[j] = 0.0f;
            for (int i = 0; i < dk; ++i)
                for (int j = 0; j < dv; ++j) o[j] += qt[i] * st[i * dv + j];
        }
    });
}

// ---- GatedDeltaRule::chunked, f32 (delta_rule.rs:223-310) -----------------
int chunked_f32(const gdr_oracle_batch* b, const float* q, const float* k, const float* v,
                const float* g, const float* beta, const float* state_in, float* out,
                float* state_out) {
    View<float> at{*b};
    const int dk = b->d_k, dv = b->d_v, c = b->chunk_size;
    if (c <= 0) return 1;  // :233 "a chunk of at least one position"
    return for_pairs(b, [&](int s, int h) {
        float* st = state_out + at.state(s, h);
        if (state_in)
            std::memmove(st, state_in + at.state(s, h), sizeof(float) * dk * dv);
        else
            std::fill(st, st + dk * dv, 0.0f);
        const int t0 = b->cu_seqlens[s], len = b->cu_seqlens[s + 1] - t0;
        const int n = (len + c - 1) / c;  // :238-239
        // One chunk's working set, [C, .] row-major.
        std::vector<float> qc(c * dk), kc(c * dk), vb(c * dv), kb(c * dk), cum(c), bt(c);
        std::vector<float> pair(c * c), system(c * c), intra(c * c), a(c * c), nxt(c);
        std::vector<float> u(c * dv), w(c * dk), vnew(c * dv), o(c * dv), upd(dk * dv);
        for (int ci = 0; ci < n; ++ci) {
            // Padded to whole chunks with zeros (:241-262).
            for (int r = 0; r < c; ++r) {
                const int pos = ci * c + r;
                if (pos < len) {
                    const int64_t t = t0 + pos;
                    prepare_vec(q + at.row_qk(t, h), dk, b->l2norm_eps, true, &qc[r * dk]);
                    prepare_vec(k + at.row_qk(t, h), dk, b->l2norm_eps, false, &kc[r * dk]);
                    bt[r] = beta[at.gate(t, h)];
                    const float* vt = v + at.row_v(t, h);
                    for (int j = 0; j < dv; ++j) vb[r * dv + j] = vt[j] * bt[r];  // :266
                    cum[r] = g[at.gate(t, h)];
                } else {
                    std::fill(&qc[r * dk], &qc[r * dk] + dk, 0.0f);
                    std::fill(&kc[r * dk], &kc[r * dk] + dk, 0.0f);
                    std::fill(&vb[r * dv], &vb[r * dv] + dv, 0.0f);
                    bt[r] = 0.0f;
                    cum[r] = 0.0f;
                }
                for (int i = 0; i < dk; ++i) kb[r * dk + i] = kc[r * dk + i] * bt[r];  // :267
            }
            for (int r = 1; r < c; ++r) cum[r] += cum[r - 1];  // :272 cumsum
            // :273-276 pairwise decay exp(cum_i - cum_j), zero above the diagonal.
            for (int i = 0; i < c; ++i)
                for (int j = 0; j < c; ++j)
                    pair[i * c + j] = j <= i ? std::exp(cum[i] - cum[j]) : 0.0f;
            // :278-279 system = (k_beta k^T) o pairwise; intra = (q k^T) o pairwise.
            for (int i = 0; i < c; ++i)
                for (int j = 0; j < c; ++j) {
                    float sk = 0, sq = 0;
                    for (int e = 0; e < dk; ++e) {
                        sk += kb[i * dk + e] * kc[j * dk + e];
                        sq += qc[i * dk + e] * kc[j * dk + e];
                    }
                    system[i * c + j] = sk * pair[i * c + j];
                    intra[i * c + j] = sq * pair[i * c + j];
                }
            // :337-351 unit_lower_inverse: a = -tril(system, -1), then row
            // forward substitution a[i, :i] += sum_j a[i, j] a[j, :i]; + I.
            for (int i = 0; i < c; ++i)
                for (int j = 0; j < c; ++j) a[i * c + j] = j < i ? -system[i * c + j] : 0.0f;
            for (int i = 1; i < c; ++i) {
                for (int m = 0; m < i; ++m) {
                    float acc = 0;
                    for (int j = 0; j < i; ++j) acc += a[i * c + j] * a[j * c + m];
                    nxt[m] = a[i * c + m] + acc;
                }
                for (int m = 0; m < i; ++m) a[i * c + m] = nxt[m];
            }
            for (int i = 0; i < c; ++i) a[i * c + i] += 1.0f;
            // :284-285 new_values = A v_beta; k_cumdecay = A (k_beta o exp(cum)).
            for (int i = 0; i < c; ++i) {
                for (int j = 0; j < dv; ++j) u[i * dv + j] = 0;
                for (int e = 0; e < dk; ++e) w[i * dk + e] = 0;
                for (int j = 0; j <= i; ++j) {
                    const float aij = a[i * c + j];
                    const float ce = std::exp(cum[j]);
                    for (int e = 0; e < dv; ++e) u[i * dv + e] += aij * vb[j * dv + e];
                    for (int e = 0; e < dk; ++e) w[i * dk + e] += aij * (kb[j * dk + e] * ce);
                }
            }
            // :287-291 q o exp(cum); k o exp(last - cum); chunk decay exp(last).
            const float last = cum[c - 1];
            for (int r = 0; r < c; ++r) {
                const float eq = std::exp(cum[r]), ek = std::exp(last - cum[r]);
                for (int e = 0; e < dk; ++e) {
                    qc[r * dk + e] *= eq;
                    kc[r * dk + e] *= ek;
                }
            }
            const float decay = std::exp(last);
            // :300 v_new = U - W S
            for (int r = 0; r < c; ++r) {
                for (int j = 0; j < dv; ++j) vnew[r * dv + j] = 0;
                for (int e = 0; e < dk; ++e) {
                    const float we = w[r * dk + e];
                    const float* srow = st + e * dv;
                    for (int j = 0; j < dv; ++j) vnew[r * dv + j] += we * srow[j];
                }
                for (int j = 0; j < dv; ++j) vnew[r * dv + j] = u[r * dv + j] - vnew[r * dv + j];
            }
            // :301 o = q S + intra v_new
            for (int r = 0; r < c; ++r) {
                float* orow = &o[r * dv];
                for (int j = 0; j < dv; ++j) orow[j] = 0;
                for (int e = 0; e < dk; ++e) {
                    const float qe = qc[r * dk + e];
                    const float* srow = st + e * dv;
                    for (int j = 0; j < dv; ++j) orow[j] += qe * srow[j];
                }
                for (int j2 = 0; j2 <= r; ++j2) {
                    const float ie = intra[r * c + j2];
                    for (int j = 0; j < dv; ++j) orow[j] += ie * vnew[j2 * dv + j];
                }
            }
            // :302 S = S * decay + k^T v_new
            for (int e = 0; e < dk * dv; ++e) upd[e] = 0;
            for (int r = 0; r < c; ++r)
                for (int e = 0; e < dk; ++e) {
                    const float ke = kc[r * dk + e];
                    for (int j = 0; j < dv; ++j) upd[e * dv + j] += ke * vnew[r * dv + j];
                }
            for (int e = 0; e < dk * dv; ++e) st[e] = st[e] * decay + upd[e];
            // :304-309 the padding sliced off.
            for (int r = 0; r < c && ci * c + r < len; ++r) {
                float* dst = out + at.row_v(t0 + ci * c + r, h);
                std::memcpy(dst, &o[r * dv], sizeof(float) * dv);
            }
        }
    });
}

}  // namespace

extern "C" {

int gdr_oracle_scalar_f64(const gdr_oracle_batch* b, const double* q, const double* k,
                          const double* v, const double* g, const double* beta,
                          const double* state_in, double* out, double* state_out) {
    if (!valid(b)) return 1;
    return scalar_f64(b, q, k, v, g, beta, state_in, out, state_out);
}

int gdr_oracle_recurrent(const gdr_oracle_batch* b, const float* q, const float* k,
                         const float* v, const float* g, const float* beta,
                         const float* state_in, float* out, float* state_out) {
    if (!valid(b)) return 1;
    return recurrent_f32(b, q, k, v, g, beta, state_in, out, state_out);
}

int gdr_oracle_chunked(const gdr_oracle_batch* b, const float* q, const float* k,
                       const float* v, const float* g, const float* beta,
                       const float* state_in, float* out, float* state_out) {
    if (!valid(b)) return 1;
    return chunked_f32(b, q, k, v, g, beta, state_in, out, state_out);
}

int gdr_oracle_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
