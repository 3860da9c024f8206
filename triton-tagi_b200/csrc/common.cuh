// Internal helpers shared by the libtagi_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tagi_b200.h"

namespace tagi {

// Records a printf-style message for tagi_last_error() on the calling thread.
void set_error(const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Counts one kernel launch and converts a pending launch/runtime error into
// TAGI_E_LAUNCH with a message. Every launch site calls it exactly once.
int check_launch(const char* what);

// Row-split index map: i -> (i / div) * outer + (i % div) * stride (div <= 0: i * stride).
struct RowMap {
    int64_t div, outer, stride;
    __host__ __device__ __forceinline__ int64_t off(int64_t i) const {
        if (div <= 0) return i * stride;
        const uint32_t q = static_cast<uint32_t>(i) / static_cast<uint32_t>(div);
        const uint32_t r = static_cast<uint32_t>(i) - q * static_cast<uint32_t>(div);
        return static_cast<int64_t>(q) * outer + static_cast<int64_t>(r) * stride;
    }
};

inline RowMap plain_rows(int64_t stride) { return RowMap{0, 0, stride}; }

// Capped closed-form update of one (mean, variance) pair, as
// triton_tagi/update/parameters.py:77-93: the bound is sqrt(max(S,1e-10))/cap,
// each delta is clipped to it with its sign kept (sign(0) = 0), and a
// variance that would become non-positive is floored to 1e-5.
__device__ __forceinline__ void capped_pair(float& m, float& S, float dm, float dS, float cap) {
    const float bound = sqrtf(fmaxf(S, 1e-10f)) / cap;
    const float sm = dm > 0.f ? 1.f : (dm < 0.f ? -1.f : 0.f);
    const float sS = dS > 0.f ? 1.f : (dS < 0.f ? -1.f : 0.f);
    m = m + sm * fminf(fabsf(dm), bound);
    const float S_raw = S + sS * fminf(fabsf(dS), bound);
    S = S_raw <= 0.f ? 1e-5f : S_raw;
}

// Rectified-Gaussian moments of a = max(0, z), z ~ N(mz, Sz), and the Jacobian
// J = Phi(alpha), alpha = mz / sqrt(Sz) (triton_tagi/layers/relu.py:63-86).
//
// The reference evaluates
//   mu = s phi + mz Phi,  var = -mu^2 + 2 mu mz - mz s phi + (Sz - mz^2) Phi
// with Phi = (1 + erf(alpha/sqrt2))/2, and for alpha < -5 with the leading
// asymptotic term Phi = phi/|alpha|. For negative alpha the terms of var cancel
// (by a factor of ~1e3 near alpha = -4) and 1 + erf loses most of Phi's digits,
// so two float32 evaluations of that form differ in the leading digits of
// small variances. Here the same moments are written through the Mills ratio
// R(t) = (1 - Phi(t)) / phi(t) of t = |alpha| and the two functions
// u(t) = 1 - t R(t), w(t) = R(t) - t u(t), each positive on t >= 0:
//   alpha < 0:  mu = s phi u,       var = Sz phi (w - phi u^2),            J = phi R
//   alpha >= 0: mu = mz + s phi u,  var = Sz (1 - phi (w + 2 alpha u + phi u^2)),
//               J = 1 - phi R
// (substituting Phi = phi R or 1 - phi R into the reference's expressions), so
// no term cancels. R, u and w are evaluated as three numerators of degree 5 in
// t over one common denominator of degree 5, on [0, 8] (|t| beyond 8 only
// meets phi < 1e-14), fitted for this library to the functions' definitions by
// weighted least squares (relative error below 4e-7, 5e-7 evaluated in
// float32). The reference's asymptotic branch is kept
// for alpha < -5 and simplified exactly: with Phi = phi/|alpha| its mu is 0 and
// its var is Sz phi / |alpha|.
__device__ __forceinline__ float poly5(const float (&c)[6], float t) {
    float a = c[5];
#pragma unroll
    for (int i = 4; i >= 0; --i) a = fmaf(a, t, c[i]);
    return a;
}

// The shared core: (mu, var, Phi) through the Mills-ratio forms above, without
// the reference ReLU's alpha < -5 branch; returns alpha and phi(alpha).
// EXACT_EXP evaluates phi with expf instead of the hardware approximation
// (about 1e-6 relative near |alpha| = 8); FAST_ALPHA forms alpha and sd from
// the hardware reciprocal square root instead of a correctly rounded sqrt and
// division.
struct RectGauss {
    float mu, v, cdf, alpha, pdf, Ss;
};

template <bool EXACT_EXP, bool FAST_ALPHA = false>
__device__ __forceinline__ RectGauss rect_gauss(float mz, float Sz) {
    constexpr float kInvSqrt2Pi = 0.3989422804014327f;
    constexpr float kR[6] = {1.253314207e+00f, 1.188586252e+00f, 5.311839209e-01f,
                             1.276814494e-01f, 1.468054771e-02f, -2.474966628e-08f};
    constexpr float kU[6] = {9.999996599e-01f, 4.929401602e-01f, 1.284475416e-01f,
                             1.464294732e-02f, 6.302450154e-07f, 1.128922133e-08f};
    constexpr float kW[6] = {1.253314576e+00f, 1.885815760e-01f, 3.825437504e-02f,
                             -7.732495484e-04f, 3.961302328e-05f, -9.044357008e-07f};
    constexpr float kQ[6] = {1.0f, 1.746248240e+00f, 1.317049340e+00f,
                             5.458146858e-01f, 1.276858994e-01f, 1.468004551e-02f};
    RectGauss g;
    g.Ss = fmaxf(Sz, 1e-30f);
    float sd;
    if (FAST_ALPHA) {
        // callers without a branch on alpha: the hardware reciprocal square root
        // (a few ulp on alpha and sd)
        const float rs = rsqrtf(g.Ss);
        sd = g.Ss * rs;
        g.alpha = mz * rs;
    } else {
        sd = sqrtf(g.Ss);
        g.alpha = mz / sd;  // correctly rounded: decides the reference ReLU's branch at -5
    }
    const float e = -0.5f * g.alpha * g.alpha;
    g.pdf = (EXACT_EXP ? expf(e) : __expf(e)) * kInvSqrt2Pi;
    const float t = fminf(fabsf(g.alpha), 8.0f);
    const float iq = __frcp_rn(poly5(kQ, t));
    const float R = poly5(kR, t) * iq, u = poly5(kU, t) * iq, w = poly5(kW, t) * iq;
    const float pu = g.pdf * u;
    if (g.alpha < 0.0f) {
        g.cdf = g.pdf * R;
        g.mu = sd * pu;
        g.v = g.Ss * (g.pdf * fmaf(-pu, u, w));
    } else {
        g.cdf = fmaf(-g.pdf, R, 1.0f);
        g.mu = fmaf(sd, pu, mz);
        g.v = g.Ss * fmaf(-g.pdf, fmaf(pu, u, fmaf(2.0f * g.alpha, u, w)), 1.0f);
    }
    return g;
}

__device__ __forceinline__ void relu_one(float mz, float Sz, float& ma, float& Sa, float& J) {
    RectGauss g = rect_gauss<false>(mz, Sz);
    if (g.alpha < -5.0f) {
        g.cdf = __fdividef(g.pdf, -g.alpha);
        g.mu = 0.0f;
        g.v = g.Ss * g.cdf;
    }
    ma = g.mu;
    Sa = fmaxf(g.v, 0.0f);
    J = g.cdf;
}

constexpr int kNumSMs = 148;

inline unsigned grid_1d(int64_t n, int threads, int64_t max_blocks = 148 * 16) {
    int64_t b = (n + threads - 1) / threads;
    if (b > max_blocks) b = max_blocks;
    if (b < 1) b = 1;
    return static_cast<unsigned>(b);
}

}  // namespace tagi

#define TAGI_REQUIRE(cond, code, ...)  \
    do {                               \
        if (!(cond)) {                 \
            tagi::set_error(__VA_ARGS__); \
            return (code);             \
        }                              \
    } while (0)
