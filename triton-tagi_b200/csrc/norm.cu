// BatchNorm2D and RMSNorm moment kernels.
//
// Channel reductions run one block per channel over the (N, H*W) slab with
// float64 accumulation in a fixed order (deterministic, no atomics), so the
// sums can be all-reduced across data-parallel ranks before the statistics
// are finalised on the device.
#include "common.cuh"

namespace tagi {
namespace {

constexpr int kRedThreads = 512;

template <int NV>
__device__ __forceinline__ void block_sum(double (&v)[NV], double* smem) {
    // smem: NV * (kRedThreads / 32) doubles
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
        if (lane == 0) smem[j * 32 + warp] = v[j];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            double t = lane < nw ? smem[j * 32 + lane] : 0.0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            v[j] = t;
        }
    }
}

// sums[c] = sum mz, sums[C+c] = sum Sz, sums[2C+c] = sum mz^2 over (n, hw).
__global__ void __launch_bounds__(kRedThreads) bn_sums_kernel(const float* mz, const float* Sz,
                                                              double* sums, int N, int C, int HW) {
    __shared__ double smem[3 * 32];
    const int c = blockIdx.x;
    double v[3] = {0.0, 0.0, 0.0};
    const int64_t per = static_cast<int64_t>(N) * HW;
    for (int64_t t = threadIdx.x; t < per; t += blockDim.x) {
        const int n = static_cast<int>(t / HW), hw = static_cast<int>(t % HW);
        const int64_t o = (static_cast<int64_t>(n) * C + c) * HW + hw;
        const double m = mz[o];
        v[0] += m;
        v[1] += Sz[o];
        v[2] += m * m;
    }
    block_sum<3>(v, smem);
    if (threadIdx.x == 0) {
        sums[c] = v[0];
        sums[C + c] = v[1];
        sums[2 * C + c] = v[2];
    }
}

// batchnorm2d.py:336-355, in float32 from the float32-rounded means.
__global__ void bn_finalize_kernel(const double* sums, int C, double count, float* mean,
                                   float* var, float* rmean, float* rvar, float* mw, int first,
                                   int preserve_var, float momentum, float one_minus, float eps) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float m = static_cast<float>(sums[c] / count);
    const float mS = static_cast<float>(sums[C + c] / count);
    const float msq = static_cast<float>(sums[2 * C + c] / count);
    const float bessel = static_cast<float>(count / (count - 1.0));
    const float v = (mS + msq - m * m) * bessel;
    mean[c] = m;
    var[c] = v;
    if (rmean && rvar) {
        if (first) {
            rmean[c] = m;
            rvar[c] = v;
            if (preserve_var && mw) mw[c] = sqrtf(v + eps);
        } else {
            rmean[c] = one_minus * rmean[c] + momentum * m;
            rvar[c] = one_minus * rvar[c] + momentum * v;
        }
    }
}

// batchnorm2d.py:59-126 (same operation order).
__global__ void bn_forward_kernel(const float* mz, const float* Sz, const float* mean,
                                  const float* var, const float* mg, const float* Sg,
                                  const float* mb, const float* Sb, float* ma, float* Sa,
                                  float* mhat, float* Shat, int64_t total, int C, int HW,
                                  float eps) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>((i / HW) % C);
        const float rs = var[c];
        const float inv_std = 1.0f / sqrtf(rs + eps);
        const float m_hat = (mz[i] - mean[c]) * inv_std;
        const float S_hat = Sz[i] / (rs + eps);
        const float g = mg[c], sg = Sg[c];
        ma[i] = g * m_hat + mb[c];
        Sa[i] = g * g * S_hat + sg * m_hat * m_hat + sg * S_hat + Sb[c];
        if (mhat) mhat[i] = m_hat;
        if (Shat) Shat[i] = S_hat;
    }
}

// batchnorm2d.py:134-192 plus the gamma/beta sums of 465-482, one block per channel.
__global__ void __launch_bounds__(kRedThreads) bn_backward_kernel(
    const float* dma, const float* dSa, const float* mhat, const float* var, const float* mg,
    float* dmz, float* dSz, double* grads, int N, int C, int HW, float eps) {
    __shared__ double smem[4 * 32];
    const int c = blockIdx.x;
    const float g = mg[c];
    const float rs = var[c];
    const float inv_std = 1.0f / sqrtf(rs + eps);
    const float inv_var = 1.0f / (rs + eps);
    double v[4] = {0.0, 0.0, 0.0, 0.0};
    const int64_t per = static_cast<int64_t>(N) * HW;
    for (int64_t t = threadIdx.x; t < per; t += blockDim.x) {
        const int n = static_cast<int>(t / HW), hw = static_cast<int>(t % HW);
        const int64_t o = (static_cast<int64_t>(n) * C + c) * HW + hw;
        const float dm = dma[o], dS = dSa[o], mh = mhat[o];
        v[0] += static_cast<double>(dm * mh);
        v[1] += static_cast<double>(dS * (mh * mh));
        v[2] += dm;
        v[3] += dS;
        dmz[o] = (dm * g) * inv_std;
        dSz[o] = (dS * g * g) * inv_var;
    }
    block_sum<4>(v, smem);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) grads[j * C + c] = v[j];
    }
}

// Deltas S*g_m, S^2*g_S from float64 sums, written out or applied with the cap.
__device__ __forceinline__ void vector_apply(int64_t i, double gm, double gS, int mode, float* m,
                                             float* S, float* d_m, float* d_S, float cap) {
    const float s = S[i];
    const float dm = s * static_cast<float>(gm);
    const float dS = (s * s) * static_cast<float>(gS);
    if (mode == TAGI_WGRAD_DELTAS) {
        d_m[i] = dm;
        d_S[i] = dS;
    } else {
        float mm = m[i], ss = s;
        capped_pair(mm, ss, dm, dS, cap);
        m[i] = mm;
        S[i] = ss;
    }
}

__global__ void bn_apply_kernel(const double* grads, int C, int mode, float* mw, float* Sw,
                                float* mb, float* Sb, float* d_mw, float* d_Sw, float* d_mb,
                                float* d_Sb, float cap) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    vector_apply(c, grads[c], grads[C + c], mode, mw, Sw, d_mw, d_Sw, cap);
    vector_apply(c, grads[2 * C + c], grads[3 * C + c], mode, mb, Sb, d_mb, d_Sb, cap);
}

__global__ void vector_apply_kernel(const double* gm, const double* gS, int64_t n, int mode,
                                    float* m, float* S, float* d_m, float* d_S, float cap) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        vector_apply(i, gm[i], gS[i], mode, m, S, d_m, d_S, cap);
}

// ---- RMSNorm (rms_norm.py:93-134), one warp per row ---------------------------
__global__ void rmsnorm_fwd_kernel(const float* ma, const float* Sa, const float* mw,
                                   const float* Sw, float* mz, float* Sz, float* inv_rms,
                                   int64_t rows, int ni, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
         r < rows; r += warps) {
        const float* a = ma + r * ni;
        const float* s = Sa + r * ni;
        float acc = 0.f;
        for (int j = lane; j < ni; j += 32) acc += a[j] * a[j] + s[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const float inv = 1.0f / sqrtf(acc / static_cast<float>(ni) + eps);
        if (lane == 0) inv_rms[r] = inv;
        for (int j = lane; j < ni; j += 32) {
            const float w = mw[j], sw = Sw[j], x = a[j];
            mz[r * ni + j] = inv * x * w;
            Sz[r * ni + j] = (inv * inv) * (s[j] * (w * w + sw) + sw * x * x);
        }
    }
}

__global__ void rmsnorm_bwd_prop_kernel(const float* dmz, const float* dSz, const float* inv_rms,
                                        const float* mw, float* dma, float* dSa, int64_t total,
                                        int ni) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float t = inv_rms[i / ni] * mw[i % ni];
        dma[i] = t * dmz[i];
        dSa[i] = t * t * dSz[i];
    }
}

// Column sums over rows: block = 32 columns x 32 row-lanes.
__global__ void rmsnorm_bwd_sums_kernel(const float* dmz, const float* dSz, const float* ma,
                                        const float* inv_rms, double* sums, int64_t rows,
                                        int ni) {
    __shared__ double sm[2][32][33];
    const int col = blockIdx.x * 32 + threadIdx.x;
    double s_mu = 0.0, s_var = 0.0;
    if (col < ni) {
        for (int64_t r = threadIdx.y; r < rows; r += blockDim.y) {
            const float inv = inv_rms[r];
            const int64_t o = r * ni + col;
            const float x = ma[o];
            s_mu += static_cast<double>(inv * x * dmz[o]);
            s_var += static_cast<double>(inv * inv * x * x * dSz[o]);
        }
    }
    sm[0][threadIdx.y][threadIdx.x] = s_mu;
    sm[1][threadIdx.y][threadIdx.x] = s_var;
    __syncthreads();
    if (threadIdx.y == 0 && col < ni) {
        double a = 0.0, b = 0.0;
        for (int y = 0; y < static_cast<int>(blockDim.y); ++y) {
            a += sm[0][y][threadIdx.x];
            b += sm[1][y][threadIdx.x];
        }
        sums[col] = a;
        sums[ni + col] = b;
    }
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" int tagi_bn_channel_sums(const float* mz, const float* Sz, double* sums, int64_t N,
                                    int64_t C, int64_t HW, void* stream) {
    const char* what = "tagi_bn_channel_sums";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && sums, TAGI_E_BAD_ARG, "%s: null pointer", what);
    bn_sums_kernel<<<(unsigned)C, kRedThreads, 0, as_stream(stream)>>>(mz, Sz, sums, (int)N, (int)C,
                                                                       (int)HW);
    return check_launch(what);
}

extern "C" int tagi_bn_finalize(const double* sums, int64_t C, double count, float* mean,
                                float* var, float* running_mean, float* running_var, float* mw,
                                int first, int preserve_var, float momentum, float eps,
                                void* stream) {
    const char* what = "tagi_bn_finalize";
    TAGI_REQUIRE(C >= 0 && count > 1.0, TAGI_E_BAD_ARG, "%s: need count > 1", what);
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(sums && mean && var, TAGI_E_BAD_ARG, "%s: null pointer", what);
    const float one_minus = static_cast<float>(1.0 - static_cast<double>(momentum));
    bn_finalize_kernel<<<grid_1d(C, 128), 128, 0, as_stream(stream)>>>(
        sums, (int)C, count, mean, var, running_mean, running_var, mw, first, preserve_var,
        momentum, one_minus, eps);
    return check_launch(what);
}

extern "C" int tagi_bn_forward(const float* mz, const float* Sz, const float* mean,
                               const float* var, const float* mg, const float* Sg,
                               const float* mb, const float* Sb, float* ma, float* Sa,
                               float* m_hat, float* S_hat, int64_t N, int64_t C, int64_t HW,
                               float eps, void* stream) {
    const char* what = "tagi_bn_forward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    const int64_t total = N * C * HW;
    if (total == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && mean && var && mg && Sg && mb && Sb && ma && Sa, TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    bn_forward_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        mz, Sz, mean, var, mg, Sg, mb, Sb, ma, Sa, m_hat, S_hat, total, (int)C, (int)HW, eps);
    return check_launch(what);
}

extern "C" int tagi_bn_backward(const float* dma, const float* dSa, const float* m_hat,
                                const float* var, const float* mg, float* dmz, float* dSz,
                                double* grads, int64_t N, int64_t C, int64_t HW, float eps,
                                void* stream) {
    const char* what = "tagi_bn_backward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(dma && dSa && m_hat && var && mg && dmz && dSz && grads, TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    bn_backward_kernel<<<(unsigned)C, kRedThreads, 0, as_stream(stream)>>>(
        dma, dSa, m_hat, var, mg, dmz, dSz, grads, (int)N, (int)C, (int)HW, eps);
    return check_launch(what);
}

extern "C" int tagi_bn_apply_grads(const double* grads, int64_t C, int mode, float* mw, float* Sw,
                                   float* mb, float* Sb, float* d_mw, float* d_Sw, float* d_mb,
                                   float* d_Sb, float cap_factor, void* stream) {
    const char* what = "tagi_bn_apply_grads";
    TAGI_REQUIRE(C >= 0, TAGI_E_BAD_ARG, "%s: bad size", what);
    TAGI_REQUIRE(mode == TAGI_WGRAD_DELTAS || mode == TAGI_WGRAD_UPDATE, TAGI_E_BAD_ARG,
                 "%s: bad mode", what);
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(grads && Sw && Sb, TAGI_E_BAD_ARG, "%s: null pointer", what);
    if (mode == TAGI_WGRAD_DELTAS)
        TAGI_REQUIRE(d_mw && d_Sw && d_mb && d_Sb, TAGI_E_BAD_ARG, "%s: null delta", what);
    else
        TAGI_REQUIRE(mw && mb && cap_factor > 0.f, TAGI_E_BAD_ARG, "%s: bad update args", what);
    bn_apply_kernel<<<grid_1d(C, 128), 128, 0, as_stream(stream)>>>(
        grads, (int)C, mode, mw, Sw, mb, Sb, d_mw, d_Sw, d_mb, d_Sb, cap_factor);
    return check_launch(what);
}

extern "C" int tagi_apply_vector_sums(const double* g_m, const double* g_S, int64_t n, int mode,
                                      float* m, float* S, float* d_m, float* d_S,
                                      float cap_factor, void* stream) {
    const char* what = "tagi_apply_vector_sums";
    TAGI_REQUIRE(n >= 0, TAGI_E_BAD_ARG, "%s: bad size", what);
    TAGI_REQUIRE(mode == TAGI_WGRAD_DELTAS || mode == TAGI_WGRAD_UPDATE, TAGI_E_BAD_ARG,
                 "%s: bad mode", what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(g_m && g_S && S, TAGI_E_BAD_ARG, "%s: null pointer", what);
    if (mode == TAGI_WGRAD_DELTAS)
        TAGI_REQUIRE(d_m && d_S, TAGI_E_BAD_ARG, "%s: null delta", what);
    else
        TAGI_REQUIRE(m && cap_factor > 0.f, TAGI_E_BAD_ARG, "%s: bad update args", what);
    vector_apply_kernel<<<grid_1d(n, 256), 256, 0, as_stream(stream)>>>(g_m, g_S, n, mode, m, S,
                                                                         d_m, d_S, cap_factor);
    return check_launch(what);
}

extern "C" int tagi_rmsnorm_forward(const float* ma, const float* Sa, const float* mw,
                                    const float* Sw, float* mz, float* Sz, float* inv_rms,
                                    int64_t rows, int64_t ni, float eps, void* stream) {
    const char* what = "tagi_rmsnorm_forward";
    TAGI_REQUIRE(rows >= 0 && ni >= 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (rows == 0) return TAGI_OK;
    TAGI_REQUIRE(ma && Sa && mw && Sw && mz && Sz && inv_rms, TAGI_E_BAD_ARG, "%s: null pointer",
                 what);
    rmsnorm_fwd_kernel<<<grid_1d(rows * 32, 256), 256, 0, as_stream(stream)>>>(
        ma, Sa, mw, Sw, mz, Sz, inv_rms, rows, (int)ni, eps);
    return check_launch(what);
}

extern "C" int tagi_rmsnorm_backward(const float* dmz, const float* dSz, const float* ma,
                                     const float* inv_rms, const float* mw, float* dma,
                                     float* dSa, double* sums, int64_t rows, int64_t ni,
                                     void* stream) {
    const char* what = "tagi_rmsnorm_backward";
    TAGI_REQUIRE(rows >= 0 && ni >= 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    TAGI_REQUIRE(dmz && dSz && ma && inv_rms && mw && dma && dSa && sums, TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    cudaStream_t st = as_stream(stream);
    if (rows > 0) {
        rmsnorm_bwd_prop_kernel<<<grid_1d(rows * ni, 256), 256, 0, st>>>(dmz, dSz, inv_rms, mw,
                                                                         dma, dSa, rows * ni,
                                                                         (int)ni);
        int rc = check_launch(what);
        if (rc) return rc;
    }
    dim3 blk(32, 32);
    rmsnorm_bwd_sums_kernel<<<(unsigned)((ni + 31) / 32), blk, 0, st>>>(dmz, dSz, ma, inv_rms, sums,
                                                                        rows, (int)ni);
    return check_launch(what);
}
