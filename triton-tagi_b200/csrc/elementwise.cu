// Memory-bound elementwise and row kernels of the TAGI path.
//
// All kernels are grid-stride loops sized to a few waves of the 148 SMs; the
// flat kernels use 16-byte vector accesses when every pointer is 16-byte
// aligned and the length is a multiple of 4 (the common case for torch
// allocations), and scalar accesses otherwise.
#include <initializer_list>

#include "common.cuh"

namespace tagi {
namespace {

constexpr float kInvSqrt2Pi = 0.3989422804014327f;
constexpr float kInvSqrt2 = 0.7071067811865476f;

__host__ __device__ inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---- capped update (parameters.py:58-96) ----------------------------------
__global__ void capped_update_v4(float4* m, float4* S, const float4* dm, const float4* dS,
                                 int64_t n4, float cap) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 a = m[i], s = S[i];
        const float4 d = dm[i], e = dS[i];
        capped_pair(a.x, s.x, d.x, e.x, cap);
        capped_pair(a.y, s.y, d.y, e.y, cap);
        capped_pair(a.z, s.z, d.z, e.z, cap);
        capped_pair(a.w, s.w, d.w, e.w, cap);
        m[i] = a;
        S[i] = s;
    }
}

__global__ void capped_update_s(float* m, float* S, const float* dm, const float* dS, int64_t n,
                                float cap) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float a = m[i], s = S[i];
        capped_pair(a, s, dm[i], dS[i], cap);
        m[i] = a;
        S[i] = s;
    }
}

// ---- innovation (observation.py:24-46) -------------------------------------
__global__ void innovation_kernel(const float* y, const float* mu, const float* var, float* dmu,
                                  float* dvar, int64_t n, float sv2) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float Sy = var[i] + sv2;
        dmu[i] = (y[i] - mu[i]) / Sy;
        dvar[i] = -1.0f / Sy;
    }
}

// ---- rectified-Gaussian moments: relu_one (common.cuh) ----------------------
__global__ void relu_v4(const float4* mz, const float4* Sz, float4* ma, float4* Sa, float4* J,
                        int64_t n4) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 m = mz[i], s = Sz[i];
        float4 a, b, j;
        relu_one(m.x, s.x, a.x, b.x, j.x);
        relu_one(m.y, s.y, a.y, b.y, j.y);
        relu_one(m.z, s.z, a.z, b.z, j.z);
        relu_one(m.w, s.w, a.w, b.w, j.w);
        ma[i] = a;
        Sa[i] = b;
        J[i] = j;
    }
}

__global__ void relu_s(const float* mz, const float* Sz, float* ma, float* Sa, float* J,
                       int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        relu_one(mz[i], Sz[i], ma[i], Sa[i], J[i]);
}

// ---- Jacobian backward: dm*J, dS*J^2 ----------------------------------------
__global__ void jac_v4(const float4* dm, const float4* dS, const float4* J, float4* om,
                       float4* oS, int64_t n4) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 a = dm[i], s = dS[i], j = J[i];
        om[i] = make_float4(a.x * j.x, a.y * j.y, a.z * j.z, a.w * j.w);
        oS[i] = make_float4(s.x * j.x * j.x, s.y * j.y * j.y, s.z * j.z * j.z, s.w * j.w * j.w);
    }
}

__global__ void jac_s(const float* dm, const float* dS, const float* J, float* om, float* oS,
                      int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float j = J[i];
        om[i] = dm[i] * j;
        oS[i] = dS[i] * j * j;
    }
}

// ---- in-place add (resblock.py:69-130) ---------------------------------------
__global__ void add_v4(float4* am, float4* aS, const float4* bm, const float4* bS, int64_t n4) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 a = am[i], s = aS[i];
        const float4 b = bm[i], t = bS[i];
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
        s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
        am[i] = a;
        aS[i] = s;
    }
}

__global__ void add_s(float* am, float* aS, const float* bm, const float* bS, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        am[i] += bm[i];
        aS[i] += bS[i];
    }
}

// ---- average pooling, window = stride = k (avgpool2d.py:38-130) ------------
__global__ void avgpool_fwd_kernel(const float* ma, const float* Sa, float* om, float* oS,
                                   int64_t NC, int H, int W, int k, float inv_k2,
                                   float var_scale) {
    const int Ho = H / k, Wo = W / k;
    const int64_t total = NC * Ho * Wo;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int ow = static_cast<int>(i % Wo);
        const int oh = static_cast<int>((i / Wo) % Ho);
        const int64_t nc = i / (static_cast<int64_t>(Wo) * Ho);
        const float* pm = ma + nc * H * W + static_cast<int64_t>(oh) * k * W + ow * k;
        const float* pS = Sa + nc * H * W + static_cast<int64_t>(oh) * k * W + ow * k;
        float sm = 0.f, sS = 0.f;
        for (int kh = 0; kh < k; ++kh)
            for (int kw = 0; kw < k; ++kw) {
                sm += pm[kh * W + kw];
                sS += pS[kh * W + kw];
            }
        om[i] = sm * inv_k2;
        oS[i] = sS * var_scale;
    }
}

__global__ void avgpool_bwd_kernel(const float* dm, const float* dS, float* om, float* oS,
                                   int64_t NC, int H, int W, int k, float inv_k2,
                                   float var_scale) {
    const int Ho = H / k, Wo = W / k;
    const int64_t total = NC * H * W;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int w = static_cast<int>(i % W);
        const int h = static_cast<int>((i / W) % H);
        const int64_t nc = i / (static_cast<int64_t>(W) * H);
        const int oh = h / k, ow = w / k;
        if (oh < Ho && ow < Wo) {
            const int64_t o = nc * Ho * Wo + static_cast<int64_t>(oh) * Wo + ow;
            om[i] = dm[o] * inv_k2;
            oS[i] = dS[o] * var_scale;
        } else {
            om[i] = 0.f;
            oS[i] = 0.f;
        }
    }
}

// ---- Remax (remax.py:33-114) -------------------------------------------------
// Inputs and outputs are float32; the arithmetic runs in float64. The Remax
// closed form cancels heavily (log(1+x) of small ratios, a sum of three logs
// that nearly vanishes, exp(x)-1), so float32 evaluations that round
// differently (FMA contraction, another exp/log) disagree by up to ~1e-3 on
// its variance and Jacobian, and that difference is amplified by training: an
// MLP run whose only float64 part is Remax stays within ~1e-5 of a float64 run
// after 100 steps, against ~3e-3 for float32 Remax. Evaluating in float64
// keeps the output within the reference's own rounding error of the exact
// moments.
struct RemaxLocal {
    double Sz, mu_m, var_m, cdf;
};

__device__ __forceinline__ RemaxLocal remax_mixture(float mz_f, float Sz_f) {
    constexpr double EPS = 1e-6;
    const double mz = mz_f, Sz = Sz_f;
    RemaxLocal r;
    r.Sz = Sz;
    const double sd = sqrt(Sz);
    const double alpha = mz / sd;
    const double pdf = 0.3989422804014327 * exp(-0.5 * alpha * alpha);
    r.cdf = 0.5 + 0.5 * erf(alpha * 0.7071067811865476);
    r.mu_m = fmax(mz * r.cdf + sd * pdf, EPS);
    const double v = -r.mu_m * r.mu_m + 2.0 * r.mu_m * mz - mz * sd * pdf + (Sz - mz * mz) * r.cdf;
    r.var_m = fmax(v, EPS);
    return r;
}

struct RemaxStage2 {
    double var_log_m, cov_log, var_log_a, mu_raw;
};

__device__ __forceinline__ RemaxStage2 remax_lognormal(const RemaxLocal& l, double mu_t,
                                                       double var_log_t, double mu_log_t) {
    constexpr double EPS = 1e-6;
    RemaxStage2 s;
    s.var_log_m = log(1.0 + l.var_m / (l.mu_m * l.mu_m));
    const double mu_log_m = log(l.mu_m) - 0.5 * s.var_log_m;
    s.cov_log = log(1.0 + l.var_m / (l.mu_m * mu_t));
    const double mu_log_a = mu_log_m - mu_log_t;
    s.var_log_a = fmax(s.var_log_m + var_log_t - 2.0 * s.cov_log, 0.0);
    s.mu_raw = fmax(exp(mu_log_a + 0.5 * s.var_log_a), EPS);
    return s;
}

__device__ __forceinline__ void remax_finish(const RemaxLocal& l, const RemaxStage2& s,
                                             double sum_raw, float& ma, float& Sa, float& J) {
    constexpr double EPS = 1e-6;
    const double mu_a = s.mu_raw / sum_raw;
    const double var_a = (exp(s.var_log_a) - 1.0) * mu_a * mu_a;
    const double cov_a_m = (exp(s.var_log_m - s.cov_log) - 1.0) * mu_a * l.mu_m;
    const double cov_a_z = fmin(sqrt(var_a * l.Sz), cov_a_m / fmax(l.cdf, EPS));
    ma = static_cast<float>(mu_a);
    Sa = static_cast<float>(var_a);
    J = static_cast<float>(cov_a_z / l.Sz);
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per row, up to PER*32 classes held in registers (PER = 0: any K,
// the mixture moments are recomputed from global memory in each pass). The
// log-normal stage is recomputed in the last pass rather than stored.
template <int PER>
__global__ void remax_warp_kernel(const float* mz, const float* Sz, float* ma, float* Sa,
                                  float* J, int64_t rows, int K, int64_t stride) {
    constexpr double EPS = 1e-6;
    constexpr int R = PER > 0 ? PER : 1;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
         row < rows; row += warps) {
        const int64_t base = row * stride;
        RemaxLocal loc[R];
        double s_mu = 0.0, s_var = 0.0;
        if (PER > 0) {
#pragma unroll
            for (int p = 0; p < R; ++p) {
                const int j = lane + 32 * p;
                if (j < K) {
                    loc[p] = remax_mixture(mz[base + j], Sz[base + j]);
                    s_mu += loc[p].mu_m;
                    s_var += loc[p].var_m;
                }
            }
        } else {
            for (int j = lane; j < K; j += 32) {
                const RemaxLocal l = remax_mixture(mz[base + j], Sz[base + j]);
                s_mu += l.mu_m;
                s_var += l.var_m;
            }
        }
        const double mu_t = fmax(warp_sum(s_mu), EPS);
        const double var_t = fmax(warp_sum(s_var), EPS);
        const double var_log_t = log(1.0 + var_t / (mu_t * mu_t));
        const double mu_log_t = log(mu_t) - 0.5 * var_log_t;
        double s_raw = 0.0;
        if (PER > 0) {
#pragma unroll
            for (int p = 0; p < R; ++p) {
                const int j = lane + 32 * p;
                if (j < K) s_raw += remax_lognormal(loc[p], mu_t, var_log_t, mu_log_t).mu_raw;
            }
        } else {
            for (int j = lane; j < K; j += 32)
                s_raw += remax_lognormal(remax_mixture(mz[base + j], Sz[base + j]), mu_t,
                                         var_log_t, mu_log_t).mu_raw;
        }
        const double sum_raw = fmax(warp_sum(s_raw), EPS);
        if (PER > 0) {
#pragma unroll
            for (int p = 0; p < R; ++p) {
                const int j = lane + 32 * p;
                if (j < K) {
                    const RemaxStage2 s2 = remax_lognormal(loc[p], mu_t, var_log_t, mu_log_t);
                    remax_finish(loc[p], s2, sum_raw, ma[base + j], Sa[base + j], J[base + j]);
                }
            }
        } else {
            for (int j = lane; j < K; j += 32) {
                const RemaxLocal l = remax_mixture(mz[base + j], Sz[base + j]);
                const RemaxStage2 s2 = remax_lognormal(l, mu_t, var_log_t, mu_log_t);
                remax_finish(l, s2, sum_raw, ma[base + j], Sa[base + j], J[base + j]);
            }
        }
    }
}

// Rows of 128 < K <= kRemaxSmemK classes (attention scores): one warp per row;
// each class's mixture moments (pass 1) are computed once and kept in shared
// memory (float64), and pass 2 replaces them with the log-normal results that
// the finish needs, so nothing is evaluated twice (remax_warp_kernel<0>
// recomputes both stages from global memory). The kernel was bound by the
// float64 divisions, square roots and conversions of the XU pipe; this cuts
// the per-class transcendental work by about a quarter. A lane only touches
// its own classes (j = lane mod 32) in a fixed order; the covariance term is
// associated as ((e - 1) * mu_m / cdf) * mu_a instead of ((e - 1) * mu_a *
// mu_m) / cdf, a float64 rounding difference.
constexpr int kRemaxSmemK = 1024;
constexpr int kRemaxSmemWarps = 8;
// (two CTAs per SM fit the shared memory of K = 512; registers up to 128)
__global__ void __launch_bounds__(32 * kRemaxSmemWarps, 2)
    remax_smem_kernel(const float* mz, const float* Sz, float* ma, float* Sa, float* J,
                      int64_t rows, int K, int64_t stride) {
    constexpr double EPS = 1e-6;
    extern __shared__ double remax_rs[];  // [warp][3][K]
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double* mu_m = remax_rs + static_cast<size_t>(w) * 3 * K;
    double* var_m = mu_m + K;
    double* cdf = var_m + K;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
         row < rows; row += warps) {
        const int64_t base = row * stride;
        double s_mu = 0.0, s_var = 0.0;
        for (int j = lane; j < K; j += 32) {
            const RemaxLocal l = remax_mixture(mz[base + j], Sz[base + j]);
            mu_m[j] = l.mu_m;
            var_m[j] = l.var_m;
            cdf[j] = l.cdf;
            s_mu += l.mu_m;
            s_var += l.var_m;
        }
        const double mu_t = fmax(warp_sum(s_mu), EPS);
        const double var_t = fmax(warp_sum(s_var), EPS);
        const double var_log_t = log(1.0 + var_t / (mu_t * mu_t));
        const double mu_log_t = log(mu_t) - 0.5 * var_log_t;
        // pass 2: the log-normal stage of each class, its sum, and the factors of
        // the finish that do not depend on that sum, stored over the class's
        // three slots: mu_raw, exp(var_log_a) - 1 and
        // (exp(var_log_m - cov_log) - 1) * mu_m / max(cdf, eps)
        double s_raw = 0.0;
        for (int j = lane; j < K; j += 32) {
            RemaxLocal l;
            l.mu_m = mu_m[j];
            l.var_m = var_m[j];
            const RemaxStage2 s2 = remax_lognormal(l, mu_t, var_log_t, mu_log_t);
            s_raw += s2.mu_raw;
            const double c = fmax(cdf[j], EPS);
            mu_m[j] = s2.mu_raw;
            var_m[j] = exp(s2.var_log_a) - 1.0;
            cdf[j] = (exp(s2.var_log_m - s2.cov_log) - 1.0) * l.mu_m / c;
        }
        const double sum_raw = fmax(warp_sum(s_raw), EPS);
        // pass 3: normalise (remax_finish with the stored factors)
        for (int j = lane; j < K; j += 32) {
            const double mu_a = mu_m[j] / sum_raw;
            const double var_a = var_m[j] * mu_a * mu_a;
            const double Szd = static_cast<double>(Sz[base + j]);
            const double cov_a_z = fmin(sqrt(var_a * Szd), cdf[j] * mu_a);
            ma[base + j] = static_cast<float>(mu_a);
            Sa[base + j] = static_cast<float>(var_a);
            J[base + j] = static_cast<float>(cov_a_z / Szd);
        }
    }
}

// ---- launch helpers ---------------------------------------------------------
inline bool all_aligned(std::initializer_list<const void*> ps) {
    for (const void* p : ps)
        if (!aligned16(p)) return false;
    return true;
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" int tagi_capped_update(float* m, float* S, const float* delta_m, const float* delta_S,
                                  int64_t n, float cap_factor, void* stream) {
    const char* what = "tagi_capped_update";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: negative size", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(m && S && delta_m && delta_S, TAGI_E_BAD_ARG, "%s: null pointer", what);
    TAGI_REQUIRE(cap_factor > 0.f, TAGI_E_BAD_ARG, "%s: cap_factor must be > 0", what);
    cudaStream_t st = as_stream(stream);
    if (n % 4 == 0 && all_aligned({m, S, delta_m, delta_S}))
        capped_update_v4<<<grid_1d(n / 4, 256), 256, 0, st>>>(
            reinterpret_cast<float4*>(m), reinterpret_cast<float4*>(S),
            reinterpret_cast<const float4*>(delta_m), reinterpret_cast<const float4*>(delta_S),
            n / 4, cap_factor);
    else
        capped_update_s<<<grid_1d(n, 256), 256, 0, st>>>(m, S, delta_m, delta_S, n, cap_factor);
    return check_launch(what);
}

extern "C" int tagi_innovation(const float* y, const float* mu, const float* var, float* delta_mu,
                               float* delta_var, int64_t n, float sigma_v_sq, void* stream) {
    const char* what = "tagi_innovation";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: negative size", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(y && mu && var && delta_mu && delta_var, TAGI_E_BAD_ARG, "%s: null pointer",
                 what);
    innovation_kernel<<<grid_1d(n, 256), 256, 0, as_stream(stream)>>>(y, mu, var, delta_mu,
                                                                       delta_var, n, sigma_v_sq);
    return check_launch(what);
}

extern "C" int tagi_relu_forward(const float* mz, const float* Sz, float* ma, float* Sa, float* J,
                                 int64_t n, void* stream) {
    const char* what = "tagi_relu_forward";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: negative size", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && ma && Sa && J, TAGI_E_BAD_ARG, "%s: null pointer", what);
    cudaStream_t st = as_stream(stream);
    if (n % 4 == 0 && all_aligned({mz, Sz, ma, Sa, J}))
        relu_v4<<<grid_1d(n / 4, 256), 256, 0, st>>>(
            reinterpret_cast<const float4*>(mz), reinterpret_cast<const float4*>(Sz),
            reinterpret_cast<float4*>(ma), reinterpret_cast<float4*>(Sa),
            reinterpret_cast<float4*>(J), n / 4);
    else
        relu_s<<<grid_1d(n, 256), 256, 0, st>>>(mz, Sz, ma, Sa, J, n);
    return check_launch(what);
}

extern "C" int tagi_jacobian_backward(const float* dm, const float* dS, const float* J,
                                      float* out_m, float* out_S, int64_t n, void* stream) {
    const char* what = "tagi_jacobian_backward";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: negative size", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(dm && dS && J && out_m && out_S, TAGI_E_BAD_ARG, "%s: null pointer", what);
    cudaStream_t st = as_stream(stream);
    if (n % 4 == 0 && all_aligned({dm, dS, J, out_m, out_S}))
        jac_v4<<<grid_1d(n / 4, 256), 256, 0, st>>>(
            reinterpret_cast<const float4*>(dm), reinterpret_cast<const float4*>(dS),
            reinterpret_cast<const float4*>(J), reinterpret_cast<float4*>(out_m),
            reinterpret_cast<float4*>(out_S), n / 4);
    else
        jac_s<<<grid_1d(n, 256), 256, 0, st>>>(dm, dS, J, out_m, out_S, n);
    return check_launch(what);
}

extern "C" int tagi_add_inplace(float* a_m, float* a_S, const float* b_m, const float* b_S,
                                int64_t n, void* stream) {
    const char* what = "tagi_add_inplace";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: negative size", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(a_m && a_S && b_m && b_S, TAGI_E_BAD_ARG, "%s: null pointer", what);
    cudaStream_t st = as_stream(stream);
    if (n % 4 == 0 && all_aligned({a_m, a_S, b_m, b_S}))
        add_v4<<<grid_1d(n / 4, 256), 256, 0, st>>>(
            reinterpret_cast<float4*>(a_m), reinterpret_cast<float4*>(a_S),
            reinterpret_cast<const float4*>(b_m), reinterpret_cast<const float4*>(b_S), n / 4);
    else
        add_s<<<grid_1d(n, 256), 256, 0, st>>>(a_m, a_S, b_m, b_S, n);
    return check_launch(what);
}

extern "C" int tagi_avgpool_forward(const float* ma, const float* Sa, float* ma_out,
                                    float* Sa_out, int64_t N, int64_t C, int64_t H, int64_t W,
                                    int64_t k, float var_scale, void* stream) {
    const char* what = "tagi_avgpool_forward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && k >= 1, TAGI_E_BAD_ARG,
                 "%s: bad sizes", what);
    const int64_t total = N * C * (H / k) * (W / k);
    if (total == 0) return TAGI_OK;
    TAGI_REQUIRE(ma && Sa && ma_out && Sa_out, TAGI_E_BAD_ARG, "%s: null pointer", what);
    avgpool_fwd_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        ma, Sa, ma_out, Sa_out, N * C, (int)H, (int)W, (int)k, 1.0f / (float)(k * k), var_scale);
    return check_launch(what);
}

extern "C" int tagi_avgpool_backward(const float* dm, const float* dS, float* dm_out,
                                     float* dS_out, int64_t N, int64_t C, int64_t H, int64_t W,
                                     int64_t k, float var_scale, void* stream) {
    const char* what = "tagi_avgpool_backward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && k >= 1, TAGI_E_BAD_ARG,
                 "%s: bad sizes", what);
    const int64_t total = N * C * H * W;
    if (total == 0) return TAGI_OK;
    TAGI_REQUIRE(dm && dS && dm_out && dS_out, TAGI_E_BAD_ARG, "%s: null pointer", what);
    avgpool_bwd_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        dm, dS, dm_out, dS_out, N * C, (int)H, (int)W, (int)k, 1.0f / (float)(k * k), var_scale);
    return check_launch(what);
}

extern "C" int tagi_remax_forward(const float* mz, const float* Sz, float* ma, float* Sa,
                                  float* J, int64_t rows, int64_t K, int64_t row_stride,
                                  void* stream) {
    const char* what = "tagi_remax_forward";
    TAGI_REQUIRE(rows >= 0 && K >= 0 && row_stride >= K, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (rows == 0 || K == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && ma && Sa && J, TAGI_E_BAD_ARG, "%s: null pointer", what);
    cudaStream_t st = as_stream(stream);
    const unsigned grid = grid_1d(rows * 32, 256);
    if (K <= 32)
        remax_warp_kernel<1><<<grid, 256, 0, st>>>(mz, Sz, ma, Sa, J, rows, (int)K, row_stride);
    else if (K <= 128)
        remax_warp_kernel<4><<<grid, 256, 0, st>>>(mz, Sz, ma, Sa, J, rows, (int)K, row_stride);
    else if (K <= kRemaxSmemK) {
        static bool attr = false;
        const size_t smem = sizeof(double) * 3 * static_cast<size_t>(K) * kRemaxSmemWarps;
        if (!attr) {
            cudaFuncSetAttribute(remax_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(double) * 3 * kRemaxSmemK * kRemaxSmemWarps));
            attr = true;
        }
        remax_smem_kernel<<<grid_1d(rows * 32, 32 * kRemaxSmemWarps), 32 * kRemaxSmemWarps, smem,
                            st>>>(mz, Sz, ma, Sa, J, rows, (int)K, row_stride);
    } else
        remax_warp_kernel<0><<<grid, 256, 0, st>>>(mz, Sz, ma, Sa, J, rows, (int)K, row_stride);
    return check_launch(what);
}
