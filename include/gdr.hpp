// gdr.hpp -- a header-only C++ face of the C ABI in gdr.h, shaped like bunsen's
// Rust operator `GatedDeltaRule` (crates/public/bunsen/src/ops/transformers/
// linear_attention/delta_rule.rs:51-310): the same options (`qk_l2norm_eps`,
// `chunk_size`, defaults `Some(1e-6)` and 64), the same two forms with the same
// argument order (q, k, v, g, beta, state), and bunsen's panics as exceptions:
// a shape or option bunsen rejects (delta_rule.rs:135-150, :233) throws
// std::invalid_argument before anything launches; a CUDA-side failure throws
// std::runtime_error.
//
// Tensors are device buffers described by `View`s (pointer + dims, row-major,
// contiguous). Calls are asynchronous on `stream`; the caller owns every buffer.
#ifndef GDR_HPP
#define GDR_HPP

#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>

#include "gdr.h"

namespace bunsen_b200 {

// A contiguous device tensor: q, k [B, T, H_qk, d_k]; v, out [B, T, H_v, d_v];
// g, beta [B, T, H_v] (f32); state [B, H_v, d_k, d_v] (f32). With dtype
// GDR_DTYPE_F64 every tensor is f64, g, beta and the states included.
struct View {
    void* data = nullptr;
    int64_t dims[4] = {0, 0, 0, 0};
    int rank = 0;
};

inline View view(void* data, std::initializer_list<int64_t> dims) {
    View v;
    v.data = data;
    for (int64_t d : dims) v.dims[v.rank++] = d;
    return v;
}

struct GatedDeltaRule {
    std::optional<double> qk_l2norm_eps = 1e-6;
    int64_t chunk_size = 64;
    gdr_dtype dtype = GDR_DTYPE_BF16;  // of q, k, v and out
    gdr_algo algo = GDR_ALGO_AUTO;
    int32_t split_chunks = 0;  // segment length of GDR_ALGO_TENSOR_SPLIT; 0: chosen

    GatedDeltaRule with_qk_l2norm_eps(std::optional<double> eps) const {
        GatedDeltaRule r = *this;
        r.qk_l2norm_eps = eps;
        return r;
    }
    GatedDeltaRule with_chunk_size(int64_t c) const {
        GatedDeltaRule r = *this;
        r.chunk_size = c;
        return r;
    }

    // GatedDeltaRule::recurrent: writes `out` and `state_out`. `state` may have
    // data == nullptr (zeros).
    void recurrent(const View& q, const View& k, const View& v, const View& g, const View& beta,
                   const View& state, const View& out, const View& state_out,
                   void* stream = nullptr) const {
        run(false, q, k, v, g, beta, state, out, state_out, stream);
    }

    // GatedDeltaRule::chunked: the same arguments and results.
    void chunked(const View& q, const View& k, const View& v, const View& g, const View& beta,
                 const View& state, const View& out, const View& state_out,
                 void* stream = nullptr) const {
        if (chunk_size <= 0) throw std::invalid_argument("a chunk of at least one position");
        run(true, q, k, v, g, beta, state, out, state_out, stream);
    }

   private:
    static void expect(bool ok, const std::string& what) {
        if (!ok) throw std::invalid_argument(what);
    }

    void run(bool chunked_form, const View& q, const View& k, const View& v, const View& g,
             const View& beta, const View& state, const View& out, const View& state_out,
             void* stream) const {
        expect(q.rank == 4, "q is [B, T, H, Dk]");
        const int64_t b = q.dims[0], t = q.dims[1], h_qk = q.dims[2], d_k = q.dims[3];
        expect(k.rank == 4 && k.dims[0] == b && k.dims[1] == t && k.dims[2] == h_qk &&
                   k.dims[3] == d_k,
               "k is [B, T, H, Dk], as q");
        expect(v.rank == 4 && v.dims[0] == b && v.dims[1] == t, "v is [B, T, H, Dv]");
        const int64_t h_v = v.dims[2], d_v = v.dims[3];
        expect(h_qk > 0 && h_v % h_qk == 0, "the key heads divide the value heads");
        for (const View* x : {&g, &beta})
            expect(x->rank == 3 && x->dims[0] == b && x->dims[1] == t && x->dims[2] == h_v,
                   x == &g ? "the rule's `g` is [B, T, H]" : "the rule's `beta` is [B, T, H]");
        expect(out.rank == 4 && out.dims[0] == b && out.dims[1] == t && out.dims[2] == h_v &&
                   out.dims[3] == d_v,
               "out is [B, T, H, Dv]");
        for (const View* s : {&state, &state_out})
            expect(s->data == nullptr ||
                       (s->rank == 4 && s->dims[0] == b && s->dims[1] == h_v &&
                        s->dims[2] == d_k && s->dims[3] == d_v),
                   "the state is [B, H, Dk, Dv]");
        expect(state_out.data != nullptr, "a buffer for the final state");
        gdr_params p{};
        p.batch = static_cast<int32_t>(b);
        p.seq_len = static_cast<int32_t>(t);
        p.heads_qk = static_cast<int32_t>(h_qk);
        p.heads_v = static_cast<int32_t>(h_v);
        p.d_k = static_cast<int32_t>(d_k);
        p.d_v = static_cast<int32_t>(d_v);
        p.chunk_size = static_cast<int32_t>(chunk_size);
        p.use_l2norm = qk_l2norm_eps.has_value();
        p.l2norm_eps = qk_l2norm_eps.value_or(0.0);
        p.dtype = dtype;
        p.algo = algo;
        p.split_chunks = split_chunks;
        gdr_status st;
        if (dtype == GDR_DTYPE_F64) {
            const auto fn = chunked_form ? gdr_chunked_f64 : gdr_recurrent_f64;
            st = fn(&p, static_cast<const double*>(q.data), static_cast<const double*>(k.data),
                    static_cast<const double*>(v.data), static_cast<const double*>(g.data),
                    static_cast<const double*>(beta.data), static_cast<const double*>(state.data),
                    static_cast<double*>(out.data), static_cast<double*>(state_out.data), nullptr,
                    stream);
        } else {
            const auto fn = chunked_form ? gdr_chunked : gdr_recurrent;
            st = fn(&p, q.data, k.data, v.data, static_cast<const float*>(g.data),
                    static_cast<const float*>(beta.data), static_cast<const float*>(state.data),
                    out.data, static_cast<float*>(state_out.data), nullptr, stream);
        }
        if (st == GDR_ERR_INVALID) throw std::invalid_argument(gdr_status_string(st));
        if (st != GDR_OK) throw std::runtime_error(gdr_status_string(st));
    }
};

}  // namespace bunsen_b200

#endif  // GDR_HPP
