// The C++ face of the ABI (include/gdr.hpp): shape contracts throw like bunsen's
// panics, and on a GPU the chunked form agrees with the recurrent form (f32,
// and f64 computed in f64).
//   rule_cpp contracts   -- no GPU needed
//   rule_cpp parity      -- runs both forms on cuda:0
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "gdr.hpp"

using bunsen_b200::GatedDeltaRule;
using bunsen_b200::view;

static int contracts() {
    GatedDeltaRule rule;
    float dummy = 0.f;
    void* d = &dummy;  // never dereferenced: the checks come first
    int fails = 0;
    auto expect_throw = [&](const char* what, auto fn) {
        try {
            fn();
            std::printf("no throw: %s\n", what);
            ++fails;
        } catch (const std::invalid_argument&) {
        }
    };
    expect_throw("g shape", [&] {
        rule.chunked(view(d, {2, 5, 3, 4}), view(d, {2, 5, 3, 4}), view(d, {2, 5, 3, 6}),
                     view(d, {2, 5, 2}), view(d, {2, 5, 3}), view(nullptr, {}),
                     view(d, {2, 5, 3, 6}), view(d, {2, 3, 4, 6}));
    });
    expect_throw("zero chunk", [&] {
        rule.with_chunk_size(0).chunked(view(d, {1, 2, 1, 4}), view(d, {1, 2, 1, 4}),
                                        view(d, {1, 2, 1, 4}), view(d, {1, 2, 1}),
                                        view(d, {1, 2, 1}), view(nullptr, {}),
                                        view(d, {1, 2, 1, 4}), view(d, {1, 1, 4, 4}));
    });
    expect_throw("heads", [&] {
        rule.recurrent(view(d, {1, 2, 2, 4}), view(d, {1, 2, 2, 4}), view(d, {1, 2, 3, 4}),
                       view(d, {1, 2, 3}), view(d, {1, 2, 3}), view(nullptr, {}),
                       view(d, {1, 2, 3, 4}), view(d, {1, 3, 4, 4}));
    });
    std::printf("contracts: %s\n", fails ? "FAIL" : "ok");
    return fails ? 1 : 0;
}

static int parity() {
    const int B = 2, T = 70, Hq = 2, Hv = 4, D = 32;
    std::mt19937 gen(7);
    std::normal_distribution<float> n01;
    std::uniform_real_distribution<float> u01(0.f, 1.f);
    std::vector<float> q(B * T * Hq * D), k(q.size()), v(B * T * Hv * D), g(B * T * Hv),
        beta(g.size()), s0(B * Hv * D * D);
    for (auto& x : q) x = n01(gen);
    for (auto& x : k) x = n01(gen);
    for (auto& x : v) x = n01(gen);
    for (auto& x : g) x = -u01(gen);
    for (auto& x : beta) x = u01(gen);
    for (auto& x : s0) x = 0.1f * n01(gen);
    auto up = [](const std::vector<float>& h) {
        float* p = nullptr;
        cudaMalloc(&p, h.size() * sizeof(float));
        cudaMemcpy(p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    float *dq = up(q), *dk = up(k), *dv = up(v), *dg = up(g), *db = up(beta), *ds = up(s0);
    float *o1, *o2, *s1, *s2;
    cudaMalloc(&o1, v.size() * 4);
    cudaMalloc(&o2, v.size() * 4);
    cudaMalloc(&s1, s0.size() * 4);
    cudaMalloc(&s2, s0.size() * 4);
    GatedDeltaRule rule;
    rule.dtype = GDR_DTYPE_F32;
    rule = rule.with_chunk_size(16);
    auto Q = view(dq, {B, T, Hq, D}), K = view(dk, {B, T, Hq, D}), V = view(dv, {B, T, Hv, D});
    auto G = view(dg, {B, T, Hv}), Be = view(db, {B, T, Hv}), S = view(ds, {B, Hv, D, D});
    rule.chunked(Q, K, V, G, Be, S, view(o1, {B, T, Hv, D}), view(s1, {B, Hv, D, D}));
    rule.recurrent(Q, K, V, G, Be, S, view(o2, {B, T, Hv, D}), view(s2, {B, Hv, D, D}));
    std::vector<float> h1(v.size()), h2(v.size()), hs1(s0.size()), hs2(s0.size());
    cudaMemcpy(h1.data(), o1, h1.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(h2.data(), o2, h2.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hs1.data(), s1, hs1.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hs2.data(), s2, hs2.size() * 4, cudaMemcpyDeviceToHost);
    auto rel = [](const std::vector<float>& a, const std::vector<float>& b) {
        double m = 0, s = 0;
        for (size_t i = 0; i < a.size(); ++i) {
            m = std::fmax(m, std::fabs(a[i] - b[i]));
            s = std::fmax(s, std::fabs(b[i]));
        }
        return m / s;
    };
    const double eo = rel(h1, h2), es = rel(hs1, hs2);
    bool ok = cudaGetLastError() == cudaSuccess && eo < 1e-4 && es < 1e-4;
    std::printf("parity: out %.2e state %.2e %s\n", eo, es, ok ? "ok" : "FAIL");

    // f64: every tensor in f64 (bunsen's compute dtype for f64 inputs); both
    // forms run one kernel, so they agree exactly, and the f32 run to 1e-4.
    auto up64 = [](const std::vector<float>& h) {
        const std::vector<double> w(h.begin(), h.end());
        double* p = nullptr;
        cudaMalloc(&p, w.size() * sizeof(double));
        cudaMemcpy(p, w.data(), w.size() * sizeof(double), cudaMemcpyHostToDevice);
        return p;
    };
    double *eq = up64(q), *ek = up64(k), *ev = up64(v), *eg = up64(g), *eb = up64(beta),
           *es0 = up64(s0);
    double *p1, *p2, *t1, *t2;
    cudaMalloc(&p1, v.size() * 8);
    cudaMalloc(&p2, v.size() * 8);
    cudaMalloc(&t1, s0.size() * 8);
    cudaMalloc(&t2, s0.size() * 8);
    GatedDeltaRule r64 = rule;
    r64.dtype = GDR_DTYPE_F64;
    auto Q8 = view(eq, {B, T, Hq, D}), K8 = view(ek, {B, T, Hq, D}), V8 = view(ev, {B, T, Hv, D});
    auto G8 = view(eg, {B, T, Hv}), Be8 = view(eb, {B, T, Hv}), S8 = view(es0, {B, Hv, D, D});
    r64.chunked(Q8, K8, V8, G8, Be8, S8, view(p1, {B, T, Hv, D}), view(t1, {B, Hv, D, D}));
    r64.recurrent(Q8, K8, V8, G8, Be8, S8, view(p2, {B, T, Hv, D}), view(t2, {B, Hv, D, D}));
    std::vector<double> d1(v.size()), d2(v.size()), ds1(s0.size()), ds2(s0.size());
    cudaMemcpy(d1.data(), p1, d1.size() * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(d2.data(), p2, d2.size() * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(ds1.data(), t1, ds1.size() * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(ds2.data(), t2, ds2.size() * 8, cudaMemcpyDeviceToHost);
    const std::vector<float> f1(d1.begin(), d1.end()), fs1(ds1.begin(), ds1.end());
    const double e64o = rel(f1, h2), e64s = rel(fs1, hs2);
    const bool ok64 = cudaGetLastError() == cudaSuccess && d1 == d2 && ds1 == ds2 &&
                      e64o < 1e-4 && e64s < 1e-4;
    std::printf("f64: forms equal %d, against f32 out %.2e state %.2e %s\n",
                static_cast<int>(d1 == d2 && ds1 == ds2), e64o, e64s, ok64 ? "ok" : "FAIL");
    return ok && ok64 ? 0 : 1;
}

int main(int argc, char** argv) {
    if (argc > 1 && std::strcmp(argv[1], "parity") == 0) return parity();
    return contracts();
}
