// BatchNorm2D and RMSNorm moment kernels.
//
// Channel reductions accumulate in float64 in a fixed order (deterministic, no
// atomics), so the sums can be all-reduced across data-parallel ranks before the
// statistics are finalised on the device. Each channel is reduced by a
// thread-block cluster of S = 1, 2, 4 or 8 blocks (about 512 blocks in all):
// block j takes images j, j+S, ..., and the cluster's first block adds the S
// partial sums from its peers' shared memory in rank order. No workspace, one
// launch.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace tagi {
namespace {

constexpr int kBnThreads = 256;

// Blocks per channel: about 512 blocks in all, at most 8 and at most one per
// image; one (no cluster) from 256 channels up, where a second block per channel
// saved less than the cluster barriers cost (backward at 256 channels of 8 x 8,
// batch 128: 12.9 -> 11.3 us with one block).
int bn_split(int64_t C, int64_t N) {
    if (C >= 256) return 1;
    int s = 1;
    while (s < 8 && C * s < 512 && s < N) s *= 2;
    return s;
}

// Sums v over the block (fixed order), then over the cluster's blocks in rank
// order; the totals are valid in thread 0 of cluster rank 0. CL = false: a
// launch without clusters (one block per channel); the same sums, 0 + the
// block's total as a one-block cluster gives, with no cluster barriers.
template <int NV, bool CL = true>
__device__ __forceinline__ void cluster_channel_sum(double (&v)[NV], double* red, double* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
        if (lane == 0) red[j * 32 + warp] = v[j];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            double t = 0.0;
            for (int w = 0; w < nw; ++w) t += red[j * 32 + w];
            part[j] = t;
            if (!CL) v[j] = 0.0 + t;
        }
    }
    if constexpr (!CL) return;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0 && threadIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] = 0.0;
        for (unsigned r = 0; r < cluster.num_blocks(); ++r) {
            const double* peer = cluster.map_shared_rank(part, r);
#pragma unroll
            for (int j = 0; j < NV; ++j) v[j] += peer[j];
        }
    }
    cluster.sync();  // peers keep their shared memory until it has been read
}

template <typename K, typename... Args>
int launch_cluster(K kernel, int S, int C, cudaStream_t st, const char* what, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S), static_cast<unsigned>(C), 1);
    cfg.blockDim = dim3(kBnThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(S);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: launch failed (%s)", what, cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    return check_launch(what);
}

// S > 1: the cluster launch of `clustered`; S == 1 (one block per channel): a
// plain launch of `single`, the same kernel built without cluster barriers.
template <typename K, typename... Args>
int launch_split(K clustered, K single, int S, int C, cudaStream_t st, const char* what,
                 Args... args) {
    if (S > 1) return launch_cluster(clustered, S, C, st, what, args...);
    single<<<dim3(1u, static_cast<unsigned>(C), 1u), kBnThreads, 0, st>>>(args...);
    return check_launch(what);
}

// Elements of channel c handled by cluster block j of S: images j, j+S, ...,
// visited 4 at a time along H*W when the planes allow 16-byte access.
struct ChanSlab {
    int n0, S, nimg, HW, C, c;
    __device__ ChanSlab(int N, int C_, int HW_, int c_) : C(C_), HW(HW_), c(c_) {
        n0 = blockIdx.x;
        S = gridDim.x;
        nimg = n0 < N ? (N - n0 + S - 1) / S : 0;
    }
    __device__ __forceinline__ int64_t offset(int li, int hw) const {
        return (static_cast<int64_t>(n0 + li * S) * C + c) * HW + hw;
    }
};

// sums[c] = sum mz, sums[C+c] = sum Sz, sums[2C+c] = sum mz^2 over (n, hw).
template <bool V4, bool CL>
__global__ void __launch_bounds__(kBnThreads) bn_sums_kernel(const float* mz, const float* Sz,
                                                             double* sums, int N, int C, int HW) {
    __shared__ double red[3 * 32];
    __shared__ double part[3];
    const ChanSlab sl(N, C, HW, blockIdx.y);
    double v[3] = {0.0, 0.0, 0.0};
    if (V4) {
        // four float4 runs per thread and iteration, loaded before any is summed
        // (the same summation order as one at a time)
        constexpr int kRuns = 4;
        const int HW4 = HW / 4, total = sl.nimg * HW4;
        for (int t = threadIdx.x; t < total; t += kRuns * blockDim.x) {
            float4 m[kRuns], S[kRuns];
#pragma unroll
            for (int u = 0; u < kRuns; ++u) {
                const int tu = t + u * blockDim.x;
                if (tu < total) {
                    const int li = tu / HW4, h = (tu - li * HW4) * 4;
                    const int64_t o = sl.offset(li, h);
                    m[u] = __ldg(reinterpret_cast<const float4*>(mz + o));
                    S[u] = __ldg(reinterpret_cast<const float4*>(Sz + o));
                }
            }
#pragma unroll
            for (int u = 0; u < kRuns; ++u) {
                if (t + u * static_cast<int>(blockDim.x) >= total) break;
                const float mm[4] = {m[u].x, m[u].y, m[u].z, m[u].w};
                const float ss[4] = {S[u].x, S[u].y, S[u].z, S[u].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const double x = mm[e];
                    v[0] += x;
                    v[1] += ss[e];
                    v[2] += x * x;
                }
            }
        }
    } else {
        const int total = sl.nimg * HW;
        for (int t = threadIdx.x; t < total; t += blockDim.x) {
            const int li = t / HW;
            const int64_t o = sl.offset(li, t - li * HW);
            const double x = mz[o];
            v[0] += x;
            v[1] += Sz[o];
            v[2] += x * x;
        }
    }
    cluster_channel_sum<3, CL>(v, red, part);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        sums[sl.c] = v[0];
        sums[C + sl.c] = v[1];
        sums[2 * C + sl.c] = v[2];
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
        const float S_hat = Sz[i] * (1.0f / (rs + eps));
        const float g = mg[c], sg = Sg[c];
        ma[i] = g * m_hat + mb[c];
        Sa[i] = g * g * S_hat + sg * m_hat * m_hat + sg * S_hat + Sb[c];
        if (mhat) mhat[i] = m_hat;
        if (Shat) Shat[i] = S_hat;
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

// vector_apply's update with the parameter's current mean m and variance s
// already in registers.
__device__ __forceinline__ void update_from(int64_t i, double gm, double gS, float m, float s,
                                            float* pm, float* pS, float cap) {
    const float dm = s * static_cast<float>(gm);
    const float dS = (s * s) * static_cast<float>(gS);
    float mm = m, ss = s;
    capped_pair(mm, ss, dm, dS, cap);
    pm[i] = mm;
    pS[i] = ss;
}

// batchnorm2d.py:134-192 plus the gamma/beta sums of 465-482, one cluster per channel.
// SUMS: also the channel sums of the outgoing deltas (written to dsums[c] and
// dsums[C + c]): the bias sums of a convolution whose outputs this layer
// normalised (through a ReLU or not), which then need no pass of their own.
template <bool V4, bool SUMS, bool CL>
__global__ void __launch_bounds__(kBnThreads) bn_backward_kernel(
    const float* dma, const float* dSa, const float* mhat, const float* var, float* mg,
    float* dmz, float* dSz, const float* rj, double* grads, double* dsums, int N, int C, int HW,
    float eps, float* Sw, float* mb, float* Sb, float cap) {
    constexpr int NV = SUMS ? 6 : 4;
    __shared__ double red[NV * 32];
    __shared__ double part[NV];
    const ChanSlab sl(N, C, HW, blockIdx.y);
    const float g = mg[sl.c];
    const float rs = var[sl.c];
    // the parameters the capped update reads, loaded before the pass (only the
    // finalising thread writes them, after the cluster barriers)
    const bool fin = blockIdx.x == 0 && threadIdx.x == 0;  // cluster rank 0, thread 0
    float sw0 = 0.f, mb0 = 0.f, sb0 = 0.f;
    if (fin && cap > 0.f) {
        sw0 = Sw[sl.c];
        mb0 = mb[sl.c];
        sb0 = Sb[sl.c];
    }
    const float inv_std = 1.0f / sqrtf(rs + eps);
    const float inv_var = 1.0f / (rs + eps);
    double v[NV] = {};
    // rj: Jacobian of the ReLU that produced this layer's input (NULL: none);
    // applied to the outgoing deltas in the ReLU backward's own order.
    auto one = [&](float dm, float dS, float mh, float j, float& om, float& oS) {
        v[0] += static_cast<double>(dm * mh);
        v[1] += static_cast<double>(dS * (mh * mh));
        v[2] += dm;
        v[3] += dS;
        om = (dm * g) * inv_std;
        oS = (dS * g * g) * inv_var;
        if (rj) {
            om = om * j;
            oS = oS * j * j;
        }
        if (SUMS) {
            v[NV - 2] += om;
            v[NV - 1] += oS;
        }
    };
    if (V4) {
        // two float4 runs per thread and iteration, loaded before either is
        // used (the same summation order as one at a time)
        const int HW4 = HW / 4, total = sl.nimg * HW4;
        auto off4 = [&](int t) {
            const int li = t / HW4;
            return sl.offset(li, (t - li * HW4) * 4);
        };
        for (int t = threadIdx.x; t < total; t += 2 * blockDim.x) {
            const int t1 = t + blockDim.x;
            const bool two = t1 < total;
            const int64_t o[2] = {off4(t), two ? off4(t1) : off4(t)};
            float4 a[2], b[2], c[2], j[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                a[u] = __ldg(reinterpret_cast<const float4*>(dma + o[u]));
                b[u] = __ldg(reinterpret_cast<const float4*>(dSa + o[u]));
                c[u] = __ldg(reinterpret_cast<const float4*>(mhat + o[u]));
                j[u] = rj ? __ldg(reinterpret_cast<const float4*>(rj + o[u])) : float4{};
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                if (u == 1 && !two) break;
                float4 om, oS;
                one(a[u].x, b[u].x, c[u].x, j[u].x, om.x, oS.x);
                one(a[u].y, b[u].y, c[u].y, j[u].y, om.y, oS.y);
                one(a[u].z, b[u].z, c[u].z, j[u].z, om.z, oS.z);
                one(a[u].w, b[u].w, c[u].w, j[u].w, om.w, oS.w);
                *reinterpret_cast<float4*>(dmz + o[u]) = om;
                *reinterpret_cast<float4*>(dSz + o[u]) = oS;
            }
        }
    } else {
        const int total = sl.nimg * HW;
        for (int t = threadIdx.x; t < total; t += blockDim.x) {
            const int li = t / HW;
            const int64_t o = sl.offset(li, t - li * HW);
            one(dma[o], dSa[o], mhat[o], rj ? rj[o] : 0.f, dmz[o], dSz[o]);
        }
    }
    cluster_channel_sum<NV, CL>(v, red, part);
    if (fin) {
#pragma unroll
        for (int j = 0; j < 4; ++j) grads[j * C + sl.c] = v[j];
        if (SUMS) {
            dsums[sl.c] = v[4];
            dsums[C + sl.c] = v[5];
        }
        // cap > 0: the capped update of this channel's gamma/beta from the sums
        // (as tagi_bn_apply_grads); every block of the cluster read gamma before
        // the cluster-wide reduction above
        if (cap > 0.f) {
            update_from(sl.c, v[0], v[1], g, sw0, mg, Sw, cap);
            update_from(sl.c, v[2], v[3], mb0, sb0, mb, Sb, cap);
        }
    }
}

// The same, 4 elements of one channel plane per thread (H*W a multiple of 4).
__global__ void bn_forward_v4_kernel(const float4* mz, const float4* Sz, const float* mean,
                                     const float* var, const float* mg, const float* Sg,
                                     const float* mb, const float* Sb, float4* ma, float4* Sa,
                                     float4* mhat, float4* Shat, int64_t total4, int C, int HW4,
                                     float eps) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>((i / HW4) % C);
        const float rs = var[c], mu = mean[c];
        const float inv_std = 1.0f / sqrtf(rs + eps);
        const float inv_var = 1.0f / (rs + eps);
        const float g = mg[c], sg = Sg[c], b = mb[c], sb = Sb[c];
        const float4 m = mz[i], S = Sz[i];
        const float mv[4] = {m.x, m.y, m.z, m.w}, Sv[4] = {S.x, S.y, S.z, S.w};
        float om[4], oS[4], mh[4], Sh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            mh[e] = (mv[e] - mu) * inv_std;
            Sh[e] = Sv[e] * inv_var;
            om[e] = g * mh[e] + b;
            oS[e] = g * g * Sh[e] + sg * mh[e] * mh[e] + sg * Sh[e] + sb;
        }
        ma[i] = make_float4(om[0], om[1], om[2], om[3]);
        Sa[i] = make_float4(oS[0], oS[1], oS[2], oS[3]);
        if (mhat) mhat[i] = make_float4(mh[0], mh[1], mh[2], mh[3]);
        if (Shat) Shat[i] = make_float4(Sh[0], Sh[1], Sh[2], Sh[3]);
    }
}

// The normalised affine of the elements of one channel slab (batchnorm2d.py:
// 59-126), 4 at a time when V4, with an optional residual stream added to the
// outputs; mean mu, variance rs and scale g of the channel given.
template <bool V4>
__device__ __forceinline__ void bn_normalize(const ChanSlab& sl, const float* mz, const float* Sz,
                                             float mu, float rs, float g, float sg, float b,
                                             float sb, float* ma, float* Sa, float* mhat,
                                             const float* add_m, const float* add_S, int total,
                                             int HW4, int HW, float eps) {
    const float inv_std = 1.0f / sqrtf(rs + eps);
    const float inv_var = 1.0f / (rs + eps);
    auto off4 = [&](int t) {
        const int li = t / HW4;
        return sl.offset(li, (t - li * HW4) * 4);
    };
    for (int t = threadIdx.x; V4 && t < total; t += 2 * blockDim.x) {
        const int t1 = t + blockDim.x;
        const bool two = t1 < total;
        const int64_t o[2] = {off4(t), two ? off4(t1) : off4(t)};
        float4 m[2], S[2], am[2], aS[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            m[u] = __ldg(reinterpret_cast<const float4*>(mz + o[u]));
            S[u] = __ldg(reinterpret_cast<const float4*>(Sz + o[u]));
            if (add_m) {  // a residual stream added to the outputs
                am[u] = __ldg(reinterpret_cast<const float4*>(add_m + o[u]));
                aS[u] = __ldg(reinterpret_cast<const float4*>(add_S + o[u]));
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;
            const float mv[4] = {m[u].x, m[u].y, m[u].z, m[u].w};
            const float Sv[4] = {S[u].x, S[u].y, S[u].z, S[u].w};
            float om[4], oS[4], mh[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                mh[e] = (mv[e] - mu) * inv_std;
                const float Sh = Sv[e] * inv_var;
                om[e] = g * mh[e] + b;
                oS[e] = g * g * Sh + sg * mh[e] * mh[e] + sg * Sh + sb;
            }
            if (add_m) {
                om[0] += am[u].x; om[1] += am[u].y; om[2] += am[u].z; om[3] += am[u].w;
                oS[0] += aS[u].x; oS[1] += aS[u].y; oS[2] += aS[u].z; oS[3] += aS[u].w;
            }
            *reinterpret_cast<float4*>(ma + o[u]) = make_float4(om[0], om[1], om[2], om[3]);
            *reinterpret_cast<float4*>(Sa + o[u]) = make_float4(oS[0], oS[1], oS[2], oS[3]);
            *reinterpret_cast<float4*>(mhat + o[u]) = make_float4(mh[0], mh[1], mh[2], mh[3]);
        }
    }
    for (int t = threadIdx.x; !V4 && t < total; t += blockDim.x) {
        {
            const int li = t / HW;
            const int64_t o = sl.offset(li, t - li * HW);
            const float m_hat = (mz[o] - mu) * inv_std;
            const float S_hat = Sz[o] * inv_var;
            float om = g * m_hat + b;
            float oS = g * g * S_hat + sg * m_hat * m_hat + sg * S_hat + sb;
            if (add_m) {
                om += add_m[o];
                oS += add_S[o];
            }
            ma[o] = om;
            Sa[o] = oS;
            mhat[o] = m_hat;
        }
    }
}

// Training-mode forward in one launch (single process: no all-reduce between
// the passes): each channel's cluster sums its planes as bn_sums_kernel, rank 0
// finalises the statistics as bn_finalize_kernel (running statistics, the
// first-call scale) and hands mean, variance and scale to every rank through
// distributed shared memory, and each block normalises the elements it summed
// (read again from L2) as bn_forward_v4_kernel / bn_forward_kernel.
template <bool V4, bool CL>
__global__ void __launch_bounds__(kBnThreads) bn_train_forward_kernel(
    const float* mz, const float* Sz, float* mean, float* var, float* rmean, float* rvar,
    float* mg, const float* Sg, const float* mb, const float* Sb, float* ma, float* Sa,
    float* mhat, const float* add_m, const float* add_S, int N, int C, int HW, double count,
    int first, int preserve_var, float momentum, float one_minus, float eps) {
    __shared__ double red[3 * 32];
    __shared__ double part[3];
    __shared__ float stat[3];  // mean, variance, scale of the channel
    const ChanSlab sl(N, C, HW, blockIdx.y);
    // the channel's parameters, loaded before the first pass so that their
    // latency is not added after the cluster barriers (no launch writes them
    // but the finalising thread, which reads them first)
    const float sg = Sg[sl.c], b = mb[sl.c], sb = Sb[sl.c];
    const bool fin = blockIdx.x == 0 && threadIdx.x == 0;  // cluster rank 0, thread 0
    float g0 = 0.f, rm0 = 0.f, rv0 = 0.f;
    if (fin) {
        g0 = mg[sl.c];
        if (!first) {
            rm0 = rmean[sl.c];
            rv0 = rvar[sl.c];
        }
    }
    double v[3] = {0.0, 0.0, 0.0};
    const int HW4 = HW / 4;
    const int total = V4 ? sl.nimg * HW4 : sl.nimg * HW;
    // float4 runs: two per thread and iteration, loaded before either is summed
    // (the same summation order as one at a time)
    auto off4 = [&](int t) {
        const int li = t / HW4;
        return sl.offset(li, (t - li * HW4) * 4);
    };
    for (int t = threadIdx.x; V4 && t < total; t += 2 * blockDim.x) {
        const int t1 = t + blockDim.x;
        const bool two = t1 < total;
        const int64_t o0 = off4(t), o1 = two ? off4(t1) : o0;
        float4 m[2], S[2];
        m[0] = __ldg(reinterpret_cast<const float4*>(mz + o0));
        S[0] = __ldg(reinterpret_cast<const float4*>(Sz + o0));
        m[1] = __ldg(reinterpret_cast<const float4*>(mz + o1));
        S[1] = __ldg(reinterpret_cast<const float4*>(Sz + o1));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;
            const float mm[4] = {m[u].x, m[u].y, m[u].z, m[u].w};
            const float ss[4] = {S[u].x, S[u].y, S[u].z, S[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const double x = mm[e];
                v[0] += x;
                v[1] += ss[e];
                v[2] += x * x;
            }
        }
    }
    for (int t = threadIdx.x; !V4 && t < total; t += blockDim.x) {
        {
            const int li = t / HW;
            const int64_t o = sl.offset(li, t - li * HW);
            const double x = mz[o];
            v[0] += x;
            v[1] += Sz[o];
            v[2] += x * x;
        }
    }
    cluster_channel_sum<3, CL>(v, red, part);
    if (fin) {
        const int c = sl.c;
        const float m = static_cast<float>(v[0] / count);
        const float mS = static_cast<float>(v[1] / count);
        const float msq = static_cast<float>(v[2] / count);
        const float bessel = static_cast<float>(count / (count - 1.0));
        const float vv = (mS + msq - m * m) * bessel;
        mean[c] = m;
        var[c] = vv;
        float g = g0;
        if (first) {
            rmean[c] = m;
            rvar[c] = vv;
            if (preserve_var) {
                g = sqrtf(vv + eps);
                mg[c] = g;
            }
        } else {
            rmean[c] = one_minus * rm0 + momentum * m;
            rvar[c] = one_minus * rv0 + momentum * vv;
        }
        if constexpr (CL) {
            cg::cluster_group cluster = cg::this_cluster();
            for (unsigned r = 0; r < cluster.num_blocks(); ++r) {
                float* peer = cluster.map_shared_rank(stat, r);
                peer[0] = m;
                peer[1] = vv;
                peer[2] = g;
            }
        } else {
            stat[0] = m;
            stat[1] = vv;
            stat[2] = g;
        }
    }
    if constexpr (CL)
        cg::this_cluster().sync();
    else
        __syncthreads();
    bn_normalize<V4>(sl, mz, Sz, stat[0], stat[1], stat[2], sg, b, sb, ma, Sa, mhat, add_m,
                     add_S, total, HW4, HW, eps);
}

// Data-parallel training forward after the statistics exchange: `sums` holds
// the all-reduced [sum mz, sum Sz, sum mz^2] of every channel (the layout of
// bn_sums_kernel) over `count` elements. Every block finalises its channel with
// the arithmetic of bn_finalize_kernel (block 0 of the channel also writes the
// statistics, the running statistics and the first-call scale) and normalises
// its slab as bn_train_forward_kernel does, residual stream included: one
// launch in place of finalise, normalise and add.
template <bool V4>
__global__ void __launch_bounds__(kBnThreads) bn_sync_forward_kernel(
    const float* mz, const float* Sz, const double* sums, double count, float* mean, float* var,
    float* rmean, float* rvar, float* mg, const float* Sg, const float* mb, const float* Sb,
    float* ma, float* Sa, float* mhat, const float* add_m, const float* add_S, int N, int C,
    int HW, int first, int preserve_var, float momentum, float one_minus, float eps) {
    const ChanSlab sl(N, C, HW, blockIdx.y);
    const int c = sl.c;
    const float m = static_cast<float>(sums[c] / count);
    const float mS = static_cast<float>(sums[C + c] / count);
    const float msq = static_cast<float>(sums[2 * C + c] / count);
    const float bessel = static_cast<float>(count / (count - 1.0));
    const float vv = (mS + msq - m * m) * bessel;
    // the first call with preserve_var sets the scale; otherwise it is read
    // (no block writes it then)
    const float g = (first && preserve_var) ? sqrtf(vv + eps) : mg[c];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        mean[c] = m;
        var[c] = vv;
        if (first) {
            rmean[c] = m;
            rvar[c] = vv;
            if (preserve_var) mg[c] = g;
        } else {
            rmean[c] = one_minus * rmean[c] + momentum * m;
            rvar[c] = one_minus * rvar[c] + momentum * vv;
        }
    }
    const int HW4 = HW / 4;
    const int total = V4 ? sl.nimg * HW4 : sl.nimg * HW;
    bn_normalize<V4>(sl, mz, Sz, m, vv, g, Sg[c], mb[c], Sb[c], ma, Sa, mhat, add_m, add_S,
                     total, HW4, HW, eps);
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

// The same, 4 columns per thread (ni a multiple of 4, 16-byte aligned rows):
// thread t of a block keeps column group t % q (q = ni / 4 <= blockDim.x) and
// its gamma values and walks rows blockDim.x / q apart.
__global__ void rmsnorm_bwd_prop_v4_kernel(const float4* dmz, const float4* dSz,
                                           const float* inv_rms, const float4* mw, float4* dma,
                                           float4* dSa, int64_t rows, int q) {
    const int per = blockDim.x / q;
    if (static_cast<int>(threadIdx.x) >= per * q) return;
    const int c4 = threadIdx.x % q;
    const float4 w = mw[c4];
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * per + threadIdx.x / q; r < rows;
         r += static_cast<int64_t>(gridDim.x) * per) {
        const float inv = inv_rms[r];
        const int64_t o = r * q + c4;
        const float4 m = dmz[o], S = dSz[o];
        const float tx = inv * w.x, ty = inv * w.y, tz = inv * w.z, tw = inv * w.w;
        dma[o] = make_float4(tx * m.x, ty * m.y, tz * m.z, tw * m.w);
        dSa[o] = make_float4(tx * tx * S.x, ty * ty * S.y, tz * tz * S.z, tw * tw * S.w);
    }
}

// Column sums over rows: one cluster of S blocks per 32 columns (gridDim.y =
// column blocks); block j of a cluster takes rows j*R + ly, stepping S*R (R =
// blockDim.x / 32 row lanes, lane = column); the block's lanes are added in
// row-lane order, then the cluster's blocks in rank order (deterministic).
__global__ void __launch_bounds__(kBnThreads) rmsnorm_bwd_sums_kernel(
    const float* dmz, const float* dSz, const float* ma, const float* inv_rms, double* sums,
    int64_t rows, int ni) {
    constexpr int R = kBnThreads / 32;
    __shared__ double sm[2][R][33];
    __shared__ double part[2][32];
    const int lx = threadIdx.x & 31, ly = threadIdx.x >> 5;
    const int col = blockIdx.y * 32 + lx;
    double s_mu = 0.0, s_var = 0.0;
    if (col < ni) {
        for (int64_t r = static_cast<int64_t>(blockIdx.x) * R + ly; r < rows;
             r += static_cast<int64_t>(gridDim.x) * R) {
            const float inv = inv_rms[r];
            const int64_t o = r * ni + col;
            const float x = ma[o];
            s_mu += static_cast<double>(inv * x * dmz[o]);
            s_var += static_cast<double>(inv * inv * x * x * dSz[o]);
        }
    }
    sm[0][ly][lx] = s_mu;
    sm[1][ly][lx] = s_var;
    __syncthreads();
    if (ly == 0) {
        double a = 0.0, b = 0.0;
        for (int y = 0; y < R; ++y) {
            a += sm[0][y][lx];
            b += sm[1][y][lx];
        }
        part[0][lx] = a;
        part[1][lx] = b;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0 && ly == 0 && col < ni) {
        double a = 0.0, b = 0.0;
        for (unsigned rk = 0; rk < cluster.num_blocks(); ++rk) {
            const double* peer = cluster.map_shared_rank(&part[0][0], rk);
            a += peer[lx];
            b += peer[32 + lx];
        }
        sums[col] = a;
        sums[ni + col] = b;
    }
    cluster.sync();  // peers keep their shared memory until it has been read
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
    TAGI_REQUIRE(N * HW <= (int64_t(1) << 31) - 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    const int S = bn_split(C, N);
    const bool v4 = HW % 4 == 0 && ((reinterpret_cast<uintptr_t>(mz) | reinterpret_cast<uintptr_t>(Sz)) & 15) == 0;
    return v4 ? launch_split(bn_sums_kernel<true, true>, bn_sums_kernel<true, false>, S, (int)C,
                             as_stream(stream), what, mz, Sz, sums, (int)N, (int)C, (int)HW)
              : launch_split(bn_sums_kernel<false, true>, bn_sums_kernel<false, false>, S,
                             (int)C, as_stream(stream), what, mz, Sz, sums, (int)N, (int)C,
                             (int)HW);
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
    const uintptr_t al = reinterpret_cast<uintptr_t>(mz) | reinterpret_cast<uintptr_t>(Sz) |
                         reinterpret_cast<uintptr_t>(ma) | reinterpret_cast<uintptr_t>(Sa) |
                         reinterpret_cast<uintptr_t>(m_hat) | reinterpret_cast<uintptr_t>(S_hat);
    if (HW % 4 == 0 && (al & 15) == 0) {
        bn_forward_v4_kernel<<<grid_1d(total / 4, 256), 256, 0, as_stream(stream)>>>(
            reinterpret_cast<const float4*>(mz), reinterpret_cast<const float4*>(Sz), mean, var,
            mg, Sg, mb, Sb, reinterpret_cast<float4*>(ma), reinterpret_cast<float4*>(Sa),
            reinterpret_cast<float4*>(m_hat), reinterpret_cast<float4*>(S_hat), total / 4, (int)C,
            (int)(HW / 4), eps);
    } else {
        bn_forward_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
            mz, Sz, mean, var, mg, Sg, mb, Sb, ma, Sa, m_hat, S_hat, total, (int)C, (int)HW, eps);
    }
    return check_launch(what);
}

extern "C" int tagi_bn_train_forward(const float* mz, const float* Sz, float* mean, float* var,
                                     float* running_mean, float* running_var, float* mg,
                                     const float* Sg, const float* mb, const float* Sb, float* ma,
                                     float* Sa, float* m_hat, const float* add_m,
                                     const float* add_S, int64_t N, int64_t C, int64_t HW,
                                     int first, int preserve_var, float momentum, float eps,
                                     void* stream) {
    const char* what = "tagi_bn_train_forward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    const double count = static_cast<double>(N) * HW;
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(count > 1.0, TAGI_E_BAD_ARG, "%s: need N*H*W > 1", what);
    TAGI_REQUIRE(mz && Sz && mean && var && running_mean && running_var && mg && Sg && mb && Sb &&
                     ma && Sa && m_hat,
                 TAGI_E_BAD_ARG, "%s: null pointer", what);
    TAGI_REQUIRE((add_m == nullptr) == (add_S == nullptr), TAGI_E_BAD_ARG,
                 "%s: give both residual planes or neither", what);
    TAGI_REQUIRE(N * HW <= (int64_t(1) << 31) - 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    const int S = bn_split(C, N);
    const uintptr_t al = reinterpret_cast<uintptr_t>(mz) | reinterpret_cast<uintptr_t>(Sz) |
                         reinterpret_cast<uintptr_t>(ma) | reinterpret_cast<uintptr_t>(Sa) |
                         reinterpret_cast<uintptr_t>(m_hat) | reinterpret_cast<uintptr_t>(add_m) |
                         reinterpret_cast<uintptr_t>(add_S);
    const bool v4 = HW % 4 == 0 && (al & 15) == 0;
    const float one_minus = static_cast<float>(1.0 - static_cast<double>(momentum));
    return v4 ? launch_split(bn_train_forward_kernel<true, true>,
                             bn_train_forward_kernel<true, false>, S, (int)C, as_stream(stream),
                             what, mz, Sz, mean, var, running_mean, running_var, mg, Sg, mb, Sb,
                             ma, Sa, m_hat, add_m, add_S, (int)N, (int)C, (int)HW, count, first,
                             preserve_var, momentum, one_minus, eps)
              : launch_split(bn_train_forward_kernel<false, true>,
                             bn_train_forward_kernel<false, false>, S, (int)C, as_stream(stream),
                             what, mz, Sz, mean, var, running_mean, running_var, mg, Sg, mb, Sb,
                             ma, Sa, m_hat, add_m, add_S, (int)N, (int)C, (int)HW, count, first,
                             preserve_var, momentum, one_minus, eps);
}

extern "C" int tagi_bn_sync_forward(const float* mz, const float* Sz, const double* sums,
                                    double count, float* mean, float* var, float* running_mean,
                                    float* running_var, float* mg, const float* Sg,
                                    const float* mb, const float* Sb, float* ma, float* Sa,
                                    float* m_hat, const float* add_m, const float* add_S,
                                    int64_t N, int64_t C, int64_t HW, int first,
                                    int preserve_var, float momentum, float eps, void* stream) {
    const char* what = "tagi_bn_sync_forward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (C == 0 || N * HW == 0) return TAGI_OK;
    TAGI_REQUIRE(count > 1.0, TAGI_E_BAD_ARG, "%s: need count > 1", what);
    TAGI_REQUIRE(mz && Sz && sums && mean && var && running_mean && running_var && mg && Sg &&
                     mb && Sb && ma && Sa && m_hat,
                 TAGI_E_BAD_ARG, "%s: null pointer", what);
    TAGI_REQUIRE((add_m == nullptr) == (add_S == nullptr), TAGI_E_BAD_ARG,
                 "%s: give both residual planes or neither", what);
    TAGI_REQUIRE(N * HW <= (int64_t(1) << 31) - 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    // about 4 blocks per SM in all, each a run of whole images of one channel
    int64_t S = (4 * kNumSMs + C - 1) / C;
    S = S < 1 ? 1 : (S > N ? N : S);
    const uintptr_t al = reinterpret_cast<uintptr_t>(mz) | reinterpret_cast<uintptr_t>(Sz) |
                         reinterpret_cast<uintptr_t>(ma) | reinterpret_cast<uintptr_t>(Sa) |
                         reinterpret_cast<uintptr_t>(m_hat) | reinterpret_cast<uintptr_t>(add_m) |
                         reinterpret_cast<uintptr_t>(add_S);
    const bool v4 = HW % 4 == 0 && (al & 15) == 0;
    const float one_minus = static_cast<float>(1.0 - static_cast<double>(momentum));
    const dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>(C));
    if (v4)
        bn_sync_forward_kernel<true><<<grid, kBnThreads, 0, as_stream(stream)>>>(
            mz, Sz, sums, count, mean, var, running_mean, running_var, mg, Sg, mb, Sb, ma, Sa,
            m_hat, add_m, add_S, (int)N, (int)C, (int)HW, first, preserve_var, momentum, one_minus,
            eps);
    else
        bn_sync_forward_kernel<false><<<grid, kBnThreads, 0, as_stream(stream)>>>(
            mz, Sz, sums, count, mean, var, running_mean, running_var, mg, Sg, mb, Sb, ma, Sa,
            m_hat, add_m, add_S, (int)N, (int)C, (int)HW, first, preserve_var, momentum, one_minus,
            eps);
    return check_launch(what);
}

extern "C" int tagi_bn_backward(const float* dma, const float* dSa, const float* m_hat,
                                const float* var, float* mg, float* dmz, float* dSz,
                                const float* relu_J, double* grads, double* delta_sums,
                                int64_t N, int64_t C, int64_t HW, float eps, float* Sw, float* mb,
                                float* Sb, float cap_factor, void* stream) {
    const char* what = "tagi_bn_backward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (C == 0) return TAGI_OK;
    TAGI_REQUIRE(dma && dSa && m_hat && var && mg && dmz && dSz && grads, TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    TAGI_REQUIRE(cap_factor <= 0.f || (Sw && mb && Sb), TAGI_E_BAD_ARG,
                 "%s: the update needs Sw, mb, Sb", what);
    TAGI_REQUIRE(N * HW <= (int64_t(1) << 31) - 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    const int S = bn_split(C, N);
    const uintptr_t al = reinterpret_cast<uintptr_t>(dma) | reinterpret_cast<uintptr_t>(dSa) |
                         reinterpret_cast<uintptr_t>(m_hat) | reinterpret_cast<uintptr_t>(dmz) |
                         reinterpret_cast<uintptr_t>(dSz) | reinterpret_cast<uintptr_t>(relu_J);
    const bool v4 = HW % 4 == 0 && (al & 15) == 0;
#define TAGI_BN_BWD(V, SU)                                                                      \
    launch_split(bn_backward_kernel<V, SU, true>, bn_backward_kernel<V, SU, false>, S, (int)C,    \
                 as_stream(stream), what, dma, dSa, m_hat,                                          \
                   var, mg, dmz, dSz, relu_J, grads, delta_sums, (int)N, (int)C, (int)HW, eps, Sw, \
                   mb, Sb, cap_factor)
    const int rc = delta_sums ? (v4 ? TAGI_BN_BWD(true, true) : TAGI_BN_BWD(false, true))
                              : (v4 ? TAGI_BN_BWD(true, false) : TAGI_BN_BWD(false, false));
#undef TAGI_BN_BWD
    return rc;
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
        const int q = static_cast<int>(ni / 4);
        const uintptr_t al = reinterpret_cast<uintptr_t>(dmz) | reinterpret_cast<uintptr_t>(dSz) |
                             reinterpret_cast<uintptr_t>(mw) | reinterpret_cast<uintptr_t>(dma) |
                             reinterpret_cast<uintptr_t>(dSa);
        if (ni % 4 == 0 && q <= 256 && (al & 15) == 0) {
            const int per = 256 / q;
            rmsnorm_bwd_prop_v4_kernel<<<grid_1d((rows + per - 1) / per, 1), 256, 0, st>>>(
                reinterpret_cast<const float4*>(dmz), reinterpret_cast<const float4*>(dSz),
                inv_rms, reinterpret_cast<const float4*>(mw), reinterpret_cast<float4*>(dma),
                reinterpret_cast<float4*>(dSa), rows, q);
        } else {
            rmsnorm_bwd_prop_kernel<<<grid_1d(rows * ni, 256), 256, 0, st>>>(
                dmz, dSz, inv_rms, mw, dma, dSa, rows * ni, (int)ni);
        }
        int rc = check_launch(what);
        if (rc) return rc;
    }
    // clusters of up to 8 blocks along the rows, enough to fill the SMs
    const int64_t cblocks = (ni + 31) / 32;
    int S = 1;
    while (S < 8 && cblocks * S < 2 * kNumSMs && S * (kBnThreads / 32) < rows) S *= 2;
    TAGI_REQUIRE(cblocks <= 65535, TAGI_E_UNSUPPORTED, "%s: too many columns", what);
    return launch_cluster(rmsnorm_bwd_sums_kernel, S, static_cast<int>(cblocks), st, what, dmz,
                          dSz, ma, inv_rms, sums, rows, static_cast<int>(ni));
}
