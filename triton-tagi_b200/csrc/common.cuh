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
// J = Phi(alpha) (triton_tagi/layers/relu.py:63-86). Shared by the ReLU kernels
// and the contraction epilogues that apply a following ReLU.
__device__ __forceinline__ void relu_one(float mz, float Sz, float& ma, float& Sa, float& J) {
    constexpr float kInvSqrt2Pi = 0.3989422804014327f;
    constexpr float kInvSqrt2 = 0.7071067811865476f;
    // The kernel is bound by instruction issue, so the square root, the two
    // divisions and the exponential use the hardware approximations (a few
    // ulp, as the reference's fast sqrt, division and exp).
    const float Ss = fmaxf(Sz, 1e-30f);
    const float rs = rsqrtf(Ss);
    const float sd = Ss * rs;
    const float alpha = mz * rs;
    const float pdf = __expf(-0.5f * alpha * alpha) * kInvSqrt2Pi;
    // Below alpha = -5 the erf form cancels to 0 in fp32; the reference uses the
    // leading asymptotic term phi(alpha)/|alpha| there.
    const float cdf =
        alpha < -5.0f ? __fdividef(pdf, -alpha) : 0.5f * (1.0f + erff(alpha * kInvSqrt2));
    const float mu = sd * pdf + mz * cdf;
    const float v = -mu * mu + 2.0f * mu * mz - mz * sd * pdf + (Ss - mz * mz) * cdf;
    ma = mu;
    Sa = fmaxf(v, 0.0f);
    J = cdf;
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
