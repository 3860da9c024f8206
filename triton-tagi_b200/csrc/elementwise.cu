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

// 2 x 2 pooling of images with W a multiple of 4 (16-byte rows): per thread
// one pair of output pixels from two float4 runs of the input rows (the same
// additions, in the same order, as avgpool_fwd_kernel); 32-bit indices.
__global__ void avgpool2_fwd_v4(const float4* ma, const float4* Sa, float2* om, float2* oS,
                                uint32_t orows, uint32_t Ho, uint32_t H, uint32_t W4,
                                float inv_k2, float var_scale) {
    const uint32_t total = orows * W4;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += gridDim.x * blockDim.x) {
        const uint32_t orow = i / W4, q = i - orow * W4;  // orow = nc * Ho + oh
        const uint32_t nc = orow / Ho, oh = orow - nc * Ho;
        const uint32_t r0 = (nc * H + 2 * oh) * W4 + q;
        const float4 a = ma[r0], b = ma[r0 + W4], c = Sa[r0], d = Sa[r0 + W4];
        om[i] = make_float2((((a.x + a.y) + b.x) + b.y) * inv_k2,
                            (((a.z + a.w) + b.z) + b.w) * inv_k2);
        oS[i] = make_float2((((c.x + c.y) + d.x) + d.y) * var_scale,
                            (((c.z + c.w) + d.z) + d.w) * var_scale);
    }
}

// Its backward: each thread writes 4 input pixels of one row from a pair of
// output pixels (rows past 2 Ho get zeros, as avgpool_bwd_kernel).
__global__ void avgpool2_bwd_v4(const float2* dm, const float2* dS, float4* om, float4* oS,
                                uint32_t rows, uint32_t H, uint32_t Ho, uint32_t W4,
                                float inv_k2, float var_scale) {
    const uint32_t total = rows * W4;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += gridDim.x * blockDim.x) {
        const uint32_t row = i / W4, q = i - row * W4;  // row = nc * H + h
        const uint32_t nc = row / H, h = row - nc * H, oh = h >> 1;
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f), S = m;
        if (oh < Ho) {
            const uint32_t o = (nc * Ho + oh) * W4 + q;  // output pairs: Wo / 2 = W4 per row
            const float2 a = dm[o], b = dS[o];
            m = make_float4(a.x * inv_k2, a.x * inv_k2, a.y * inv_k2, a.y * inv_k2);
            S = make_float4(b.x * var_scale, b.x * var_scale, b.y * var_scale, b.y * var_scale);
        }
        om[i] = m;
        oS[i] = S;
    }
}

// ---- Remax (remax.py:33-114) -------------------------------------------------
// The reference evaluates, per row of K classes,
//   mixture:   m = max(E[max(0,Z)], eps), v = max(Var-expression(m), eps)
//   sums:      T = max(sum m, eps), V = max(sum v, eps)
//   log-normal: r = log(1 + v/m^2), t = log(1 + V/T^2), c = log(1 + v/(m T)),
//              mu_raw = max(exp(log m - r/2 - log T + t/2 + (r + t - 2c)/2), eps)
//   finish:    mu_a = mu_raw / max(sum mu_raw, eps), var_a = (exp(r + t - 2c) - 1) mu_a^2,
//              cov_am = (exp(r - c) - 1) mu_a m, J = min(sqrt(var_a S), cov_am / cdf) / S.
// Those exp/log pairs cancel: r + t - 2c nearly vanishes for a dominant class,
// exp(x) - 1 and log(1 + x) of small x, so float32 evaluations that round
// differently disagree in the leading digits of var_a and J (up to ~1 relative
// on attention rows). Exponentiating the logs gives exact rational forms with
// no cancelling term. With D = T - m and E = V - v (the other classes' sums,
// both >= 0) and den = m T + v:
//   mu_raw = max(m^2 (1 + V/T^2) / den, eps)
//   var_a  = mu_a^2 (v D^2 + E (m^2 + v)) / den^2
//   cov_am = mu_a v D / den
// (e.g. (1+r')(1+t')/(1+c')^2 - 1 = (v D^2 + E (m^2 + v)) / den^2 for the
// arguments r' = v/m^2, t' = V/T^2, c' = v/(m T) of the logs). Every term is
// a product or sum of non-negative factors, so float32 keeps a few ulps of
// relative accuracy; T and V are summed in float64 so that D and E (which
// subtract a class from its row's sum) keep theirs when one class dominates.
// The mixture moments come from rect_gauss (no cancelling term either). The
// kernel is issue-bound at attention sizes, so alpha, the exponential, the
// square roots and the divisions use the hardware approximations (a few ulp;
// the forms above keep that from growing). The
// reference clamps m at eps before its variance expression, which then equals
// V_true + (mu - m)(mu + m - 2 mz); that correction is applied where the
// clamp is active. The reference's clamp of the log-normal variance at 0 is
// inactive here (the form is non-negative).
struct RemaxMix {
    float m, v, cdf;
};

__device__ __forceinline__ RemaxMix remax_mixture(float mz, float Sz) {
    constexpr float EPS = 1e-6f;
    const RectGauss g = rect_gauss<false, true>(mz, Sz);
    RemaxMix r;
    r.m = fmaxf(g.mu, EPS);
    const float v = r.m == g.mu ? g.v : fmaf(g.mu - r.m, g.mu + r.m - 2.0f * mz, g.v);
    r.v = fmaxf(v, EPS);
    r.cdf = g.cdf;
    return r;
}

// Row constants after the first pass.
struct RemaxRow {
    double T, V;  // sums of m and v (clamped at eps)
    float Tf, one_t;  // T in float32 and 1 + V/T^2
};

__device__ __forceinline__ RemaxRow remax_row(double sm, double sv) {
    RemaxRow w;
    w.T = fmax(sm, 1e-6);
    w.V = fmax(sv, 1e-6);
    w.Tf = static_cast<float>(w.T);
    w.one_t = static_cast<float>(1.0 + w.V / (w.T * w.T));
    return w;
}

// Second pass of one class: mu_raw and the two factors of the finish that do
// not depend on the row sum of mu_raw.
struct RemaxFactors {
    float raw, qv, qc;
};

__device__ __forceinline__ RemaxFactors remax_factors(const RemaxMix& x, const RemaxRow& w) {
    constexpr float EPS = 1e-6f;
    const float D = static_cast<float>(fmax(w.T - static_cast<double>(x.m), 0.0));
    const float E = static_cast<float>(fmax(w.V - static_cast<double>(x.v), 0.0));
    const float den = fmaf(x.m, w.Tf, x.v);  // >= eps (v >= eps)
    const float rd = __fdividef(1.0f, den);
    RemaxFactors f;
    f.raw = fmaxf(x.m * x.m * w.one_t * rd, EPS);
    f.qv = fmaf(x.v * D, D, E * fmaf(x.m, x.m, x.v)) * rd * rd;
    f.qc = __fdividef(x.v * D * rd, fmaxf(x.cdf, EPS));
    return f;
}

// The finish of one class, with rsum = 1 / max(sum of mu_raw, eps).
__device__ __forceinline__ void remax_out(const RemaxFactors& f, float rsum, float Sz, float& ma,
                                          float& Sa, float& J) {
    const float mu_a = f.raw * rsum;
    const float var_a = mu_a * mu_a * f.qv;
    const float p = var_a * Sz;
    const float cov = fminf(p > 0.f ? p * rsqrtf(p) : 0.f, f.qc * mu_a);
    ma = mu_a;
    Sa = var_a;
    J = __fdividef(cov, Sz);
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum of one float64 value over the G warps of a row group, in warp order
// (deterministic). `red` holds G slots of this group; the barriers are
// block-wide, so every thread of the block must call this the same number of
// times.
template <int G>
__device__ __forceinline__ double group_sum(double v, double* red) {
    v = warp_sum(v);
    if (G == 1) return v;
    const int w = (threadIdx.x >> 5) % G;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < G; ++i) s += red[i];
    __syncthreads();  // the slots are written again by the next sum
    return s;
}

// G warps per row. PER > 0: the row's classes stay in registers, class
// j = (p * 32 G + t) * VEC + e for thread t < 32 G of the row's group, p < PER,
// e < VEC (VEC = 4: 16-byte accesses; needs K and the row stride multiples of 4
// and aligned pointers). PER = 0 (G = 1): any K, each pass re-reads the row
// and recomputes the mixture. Rows are visited in block-uniform steps, so the
// block barriers of group_sum are reached by every thread.
template <int PER, int VEC, int G>
__global__ void __launch_bounds__(256) remax_rows_kernel(const float* __restrict__ mz,
                                                         const float* __restrict__ Sz,
                                                         float* __restrict__ ma,
                                                         float* __restrict__ Sa,
                                                         float* __restrict__ J, int64_t rows,
                                                         int K, int64_t stride) {
    constexpr int R = PER > 0 ? PER * VEC : 1;
    constexpr int GT = 32 * G;                 // threads of a row
    constexpr int GROUPS = 256 / GT;           // rows per block step
    __shared__ double red[GROUPS][G];
    const int grp = threadIdx.x / GT, t = threadIdx.x % GT;
    float nz[R], ns[R];  // the next row's inputs (PER > 0)
    auto fetch = [&](int64_t r, float* z, float* s) {
        if (PER == 0 || r >= rows) return;
        const int64_t rb = r * stride;
#pragma unroll
        for (int p = 0; p < (PER > 0 ? PER : 1); ++p) {
            const int j0 = (p * GT + t) * VEC;
            if (j0 < K) {
                if (VEC == 4) {
                    const float4 a = *reinterpret_cast<const float4*>(mz + rb + j0);
                    const float4 b = *reinterpret_cast<const float4*>(Sz + rb + j0);
                    z[p * VEC] = a.x, z[p * VEC + 1] = a.y, z[p * VEC + 2] = a.z,
                    z[p * VEC + 3] = a.w;
                    s[p * VEC] = b.x, s[p * VEC + 1] = b.y, s[p * VEC + 2] = b.z,
                    s[p * VEC + 3] = b.w;
                } else {
                    z[p] = mz[rb + j0];
                    s[p] = Sz[rb + j0];
                }
            }
        }
    };
    fetch(static_cast<int64_t>(blockIdx.x) * GROUPS + grp, nz, ns);
    for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * GROUPS; row0 < rows;
         row0 += static_cast<int64_t>(gridDim.x) * GROUPS) {
        const int64_t row = row0 + grp;
        const bool live = row < rows;
        const int64_t base = live ? row * stride : 0;
        double sm = 0.0, sv = 0.0;
        if (PER > 0) {
            float cz[R], cs[R];
#pragma unroll
            for (int i = 0; i < R; ++i) {
                cz[i] = nz[i];
                cs[i] = ns[i];
            }
            // the next row's loads are in flight while this row is computed
            fetch(row + static_cast<int64_t>(gridDim.x) * GROUPS, nz, ns);
            RemaxMix x[R];
#pragma unroll
            for (int p = 0; p < PER; ++p) {
                if (live && (p * GT + t) * VEC < K) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        x[p * VEC + e] = remax_mixture(cz[p * VEC + e], cs[p * VEC + e]);
                        sm += x[p * VEC + e].m;
                        sv += x[p * VEC + e].v;
                    }
                }
            }
            const double tm = group_sum<G>(sm, red[grp]);
            const RemaxRow w = remax_row(tm, group_sum<G>(sv, red[grp]));
            RemaxFactors f[R];
            double sr = 0.0;
#pragma unroll
            for (int p = 0; p < PER; ++p) {
                if (live && (p * GT + t) * VEC < K) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        f[p * VEC + e] = remax_factors(x[p * VEC + e], w);
                        sr += f[p * VEC + e].raw;
                    }
                }
            }
            const float rsum =
                1.0f / static_cast<float>(fmax(group_sum<G>(sr, red[grp]), 1e-6));
#pragma unroll
            for (int p = 0; p < PER; ++p) {
                const int j0 = (p * GT + t) * VEC;
                if (live && j0 < K) {
                    float o[3][VEC];
#pragma unroll
                    for (int e = 0; e < VEC; ++e)
                        remax_out(f[p * VEC + e], rsum, cs[p * VEC + e], o[0][e], o[1][e],
                                  o[2][e]);
                    if (VEC == 4) {
                        *reinterpret_cast<float4*>(ma + base + j0) =
                            make_float4(o[0][0], o[0][1], o[0][2], o[0][3]);
                        *reinterpret_cast<float4*>(Sa + base + j0) =
                            make_float4(o[1][0], o[1][1], o[1][2], o[1][3]);
                        *reinterpret_cast<float4*>(J + base + j0) =
                            make_float4(o[2][0], o[2][1], o[2][2], o[2][3]);
                    } else {
                        ma[base + j0] = o[0][0];
                        Sa[base + j0] = o[1][0];
                        J[base + j0] = o[2][0];
                    }
                }
            }
        } else {
            static_assert(PER > 0 || G == 1, "the re-reading form runs one warp per row");
            const int lane = t;
            if (live)
                for (int j = lane; j < K; j += 32) {
                    const RemaxMix x = remax_mixture(mz[base + j], Sz[base + j]);
                    sm += x.m;
                    sv += x.v;
                }
            const RemaxRow w = remax_row(warp_sum(sm), warp_sum(sv));
            double sr = 0.0;
            if (live)
                for (int j = lane; j < K; j += 32)
                    sr += remax_factors(remax_mixture(mz[base + j], Sz[base + j]), w).raw;
            const float rsum = 1.0f / static_cast<float>(fmax(warp_sum(sr), 1e-6));
            if (live)
                for (int j = lane; j < K; j += 32) {
                    const float s = Sz[base + j];
                    remax_out(remax_factors(remax_mixture(mz[base + j], s), w), rsum, s,
                              ma[base + j], Sa[base + j], J[base + j]);
                }
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
    if (k == 2 && W % 4 == 0 && N * C * H * W < (int64_t(1) << 31) &&
        all_aligned({ma, Sa}) && ((reinterpret_cast<uintptr_t>(ma_out) |
                                    reinterpret_cast<uintptr_t>(Sa_out)) & 7) == 0) {
        const uint32_t orows = static_cast<uint32_t>(N * C * (H / 2)), W4 = static_cast<uint32_t>(W / 4);
        avgpool2_fwd_v4<<<grid_1d(static_cast<int64_t>(orows) * W4, 256), 256, 0,
                          as_stream(stream)>>>(
            reinterpret_cast<const float4*>(ma), reinterpret_cast<const float4*>(Sa),
            reinterpret_cast<float2*>(ma_out), reinterpret_cast<float2*>(Sa_out), orows,
            static_cast<uint32_t>(H / 2), static_cast<uint32_t>(H), W4, 0.25f, var_scale);
        return check_launch(what);
    }
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
    if (k == 2 && W % 4 == 0 && total < (int64_t(1) << 31) && all_aligned({dm_out, dS_out}) &&
        ((reinterpret_cast<uintptr_t>(dm) | reinterpret_cast<uintptr_t>(dS)) & 7) == 0) {
        const uint32_t rows = static_cast<uint32_t>(N * C * H), W4 = static_cast<uint32_t>(W / 4);
        avgpool2_bwd_v4<<<grid_1d(static_cast<int64_t>(rows) * W4, 256), 256, 0,
                          as_stream(stream)>>>(
            reinterpret_cast<const float2*>(dm), reinterpret_cast<const float2*>(dS),
            reinterpret_cast<float4*>(dm_out), reinterpret_cast<float4*>(dS_out), rows,
            static_cast<uint32_t>(H), static_cast<uint32_t>(H / 2), W4, 0.25f, var_scale);
        return check_launch(what);
    }
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
    const int k = static_cast<int>(K);
    const bool v4 = K % 4 == 0 && row_stride % 4 == 0 && all_aligned({mz, Sz, ma, Sa, J});
#define TAGI_REMAX(P, V, G)                                                              \
    remax_rows_kernel<P, V, G><<<grid_1d((rows + 256 / (32 * G) - 1) / (256 / (32 * G)), 1), \
                                 256, 0, st>>>(mz, Sz, ma, Sa, J, rows, k, row_stride)
    // up to 128 classes one warp per row; above, four warps per row keep the
    // registers per thread (and so the warps per SM) of a 128-class row
    if (K <= 32)
        TAGI_REMAX(1, 1, 1);
    else if (K <= 128)
        v4 ? TAGI_REMAX(1, 4, 1) : TAGI_REMAX(4, 1, 1);
    else if (K <= 512)
        v4 ? TAGI_REMAX(1, 4, 4) : TAGI_REMAX(4, 1, 4);
    else if (K <= 1024)
        v4 ? TAGI_REMAX(2, 4, 4) : TAGI_REMAX(8, 1, 4);
    else
        TAGI_REMAX(0, 1, 1);
#undef TAGI_REMAX
    return check_launch(what);
}
