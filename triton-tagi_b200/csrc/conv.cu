// Patch extraction and patch-delta gathering for the im2col Conv2D path.
//
// Layout follows the reference: patches are (N*Ho*Wo) x (C*k*k) row-major with
// row = (n, oh, ow) and column = (c, kh, kw); images are NCHW.
// padding_type 2 pads only the right/bottom edge by `padding`
// (triton_tagi/layers/conv2d.py:280-291), i.e. the top-left offset is 0.
#include <algorithm>
#include <climits>

#include "common.cuh"

namespace tagi {
namespace {

struct ConvGeom {
    int N, C, H, W, k, s, p_tl;  // p_tl: top/left padding actually applied
    int Ho, Wo;
};

bool make_geom(int64_t N, int64_t C, int64_t H, int64_t W, int64_t k, int64_t stride,
               int64_t padding, int64_t padding_type, ConvGeom* g) {
    if (N < 0 || C < 0 || H < 0 || W < 0 || k < 1 || stride < 1 || padding < 0) return false;
    if (padding_type != 1 && padding_type != 2) return false;
    const bool rb = (padding_type == 2 && padding > 0);
    const int64_t Ho = rb ? (H + padding - k) / stride + 1 : (H + 2 * padding - k) / stride + 1;
    const int64_t Wo = rb ? (W + padding - k) / stride + 1 : (W + 2 * padding - k) / stride + 1;
    if (Ho < 1 || Wo < 1) return false;
    *g = ConvGeom{(int)N, (int)C, (int)H, (int)W, (int)k, (int)stride,
                  rb ? 0 : (int)padding, (int)Ho, (int)Wo};
    return true;
}

__global__ void im2col_kernel(const float* xm, const float* xS, float* pm, float* pS,
                              ConvGeom g) {
    const int K = g.C * g.k * g.k;
    const int64_t total = static_cast<int64_t>(g.N) * g.Ho * g.Wo * K;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % K);
        const int64_t row = i / K;
        const int ow = static_cast<int>(row % g.Wo);
        const int oh = static_cast<int>((row / g.Wo) % g.Ho);
        const int n = static_cast<int>(row / (static_cast<int64_t>(g.Wo) * g.Ho));
        const int kw = col % g.k;
        const int kh = (col / g.k) % g.k;
        const int c = col / (g.k * g.k);
        const int ih = oh * g.s - g.p_tl + kh;
        const int iw = ow * g.s - g.p_tl + kw;
        float vm = 0.f, vS = 0.f;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) {
            const int64_t src = ((static_cast<int64_t>(n) * g.C + c) * g.H + ih) * g.W + iw;
            vm = xm[src];
            if (pS) vS = xS[src];
        }
        pm[i] = vm;
        if (pS) pS[i] = vS;
    }
}

// Patches with K = C*k*k a multiple of 4: one thread writes 4 consecutive
// columns of one row with a 16-byte store (a warp covers 512 contiguous bytes of
// the row), gathering the 4 inputs through L1; 32-bit index arithmetic.
__global__ void im2col_v4_kernel(const float* xm, const float* xS, float* pm, float* pS,
                                 ConvGeom g) {
    const int kk2 = g.k * g.k, K = g.C * kk2, K4 = K / 4, L = g.Ho * g.Wo;
    const int64_t total = static_cast<int64_t>(g.N) * L * K4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / K4;
        const int col = static_cast<int>(i - row * K4) * 4;
        const int n = static_cast<int>(row / L), l = static_cast<int>(row - static_cast<int64_t>(n) * L);
        const int oh = l / g.Wo, ow = l - oh * g.Wo;
        int c = col / kk2;
        const int t = col - c * kk2;
        int kh = t / g.k, kw = t - kh * g.k;
        const int64_t img = static_cast<int64_t>(n) * g.C;
        float vm[4], vS[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int ih = oh * g.s - g.p_tl + kh, iw = ow * g.s - g.p_tl + kw;
            vm[e] = vS[e] = 0.f;
            if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) {
                const int64_t src = ((img + c) * g.H + ih) * g.W + iw;
                vm[e] = __ldg(xm + src);
                if (pS) vS[e] = __ldg(xS + src);
            }
            if (++kw == g.k) {
                kw = 0;
                if (++kh == g.k) {
                    kh = 0;
                    ++c;
                }
            }
        }
        reinterpret_cast<float4*>(pm)[i] = make_float4(vm[0], vm[1], vm[2], vm[3]);
        if (pS) reinterpret_cast<float4*>(pS)[i] = make_float4(vS[0], vS[1], vS[2], vS[3]);
    }
}

// 4-byte asynchronous copy global -> shared (zero-filled when !ok): the staging
// loads of a CTA are all in flight together and waited for once.
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool ok) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src),
                 "r"(ok ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// q = i / d for 0 <= i < 2^22 and d >= 1, from the reciprocal r = 1/d: the
// fraction of (i + 0.5)/d is at least 0.5/d away from an integer and the float
// error of (i + 0.5) * r stays below that for such i.
__device__ __forceinline__ int div_small(int i, float r) {
    return static_cast<int>((static_cast<float>(i) + 0.5f) * r);
}

// Patches of one output image row (image n, output row oh) per CTA: the output
// rows r = (n, oh, 0 .. Wo-1) are Wo*K contiguous floats. The k input lines each
// channel contributes (oh*s - p + kh, all W columns) are staged in shared
// memory with asynchronous copies spread over all threads (zeros for lines
// outside the image), channel slice by channel slice; then each thread owns
// patch columns (c, kh, kw) and walks ow, so that a warp stores 32 consecutive
// columns of one patch row. Index decoding uses div_small (all indices of a CTA
// are below 2^22: staged elements and patch columns are bounded by 32 KB and K).
// PLANES: 1 (means) or 2 (means and variances).
template <int PLANES>
__global__ void im2col_rows_kernel(const float* xm, const float* xS, float* pm, float* pS,
                                   ConvGeom g, int cslice) {
    // [plane][cslice * k lines][ls]: an odd line stride puts the same column of
    // different lines (read together by a warp) in different banks
    extern __shared__ float lines[];
    const int ls = g.W | 1;
    const int n = blockIdx.x / g.Ho, oh = blockIdx.x - n * g.Ho;
    const int kk = g.k * g.k, K = g.C * kk;
    const int tid = threadIdx.x, nth = blockDim.x;
    const float rW = 1.f / g.W, rk = 1.f / g.k, rkk = 1.f / kk;
    const int64_t row0 = (static_cast<int64_t>(n) * g.Ho + oh) * g.Wo;  // first patch row
    const int ih0 = oh * g.s - g.p_tl;
    const float* img_m = xm + static_cast<int64_t>(n) * g.C * g.H * g.W;
    const float* img_S = PLANES == 2 ? xS + static_cast<int64_t>(n) * g.C * g.H * g.W : nullptr;
    for (int c0 = 0; c0 < g.C; c0 += cslice) {
        const int cs = min(cslice, g.C - c0);
        const int nlines = cs * g.k, pstride = nlines * ls;
        if (g.W % 32 == 0) {
            // a warp stages whole lines: one decode per line, lanes along the line
            for (int l = tid >> 5; l < PLANES * nlines; l += nth >> 5) {
                const int pl = PLANES == 2 && l >= nlines, li = pl ? l - nlines : l;
                const int cl = div_small(li, rk), ih = ih0 + (li - cl * g.k);
                const bool in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
                const float* src = (pl ? img_S : img_m) +
                                   (static_cast<int64_t>(c0 + cl) * g.H + (in ? ih : 0)) * g.W;
                float* dst = lines + pl * pstride + li * ls;
                for (int w = tid & 31; w < g.W; w += 32) cp_async4(dst + w, src + w, in);
            }
        } else {
            const float rn = 1.f / nlines;
            const int ne = PLANES * nlines * g.W;
            for (int e = tid; e < ne; e += nth) {
                const int line = div_small(e, rW), w = e - line * g.W;
                const int pl = PLANES == 2 ? div_small(line, rn) : 0, li = line - pl * nlines;
                const int cl = div_small(li, rk), ih = ih0 + (li - cl * g.k);
                const bool in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
                // rows outside the image are zero-filled (the source is not read)
                const float* src = (pl ? img_S : img_m) +
                                   (static_cast<int64_t>(c0 + cl) * g.H + (in ? ih : 0)) * g.W;
                cp_async4(lines + pl * pstride + li * ls + w, src + w, in);
            }
        }
        cp_async_wait_all();
        __syncthreads();
        const int ncol = cs * kk;
        // columns per thread pass and patch rows per column
        const int step = ncol >= nth ? 1 : nth / ncol;
        const int j0 = ncol >= nth ? tid : tid % ncol, ow0 = ncol >= nth ? 0 : tid / ncol;
        const int jstep = ncol >= nth ? nth : ncol;
        const int64_t ostep = static_cast<int64_t>(step) * K;
        const int istep = step * g.s;
        if (ow0 < step) {
            for (int j = j0; j < ncol; j += jstep) {
                const int cl = div_small(j, rkk), t = j - cl * kk;
                const int kh = div_small(t, rk), kw = t - kh * g.k;
                const float* line = lines + (cl * g.k + kh) * ls;
                const int64_t o0 = (row0 + ow0) * K + c0 * kk + j;
                float* om = pm + o0;
                float* oS = PLANES == 2 ? pS + o0 : nullptr;
                int iw = ow0 * g.s - g.p_tl + kw;
#pragma unroll 4
                for (int ow = ow0; ow < g.Wo; ow += step, iw += istep, om += ostep) {
                    const bool in = static_cast<unsigned>(iw) < static_cast<unsigned>(g.W);
                    *om = in ? line[iw] : 0.f;
                    if (PLANES == 2) {
                        *oS = in ? line[pstride + iw] : 0.f;
                        oS += ostep;
                    }
                }
            }
        }
        __syncthreads();
    }
}

// One thread per input pixel; taps are visited in (kh, kw) order as the
// reference does, so for identical patch inputs the sums are bit-identical.
template <bool ADJOINT>
__global__ void col2im_kernel(const float* cm, const float* cS, float* dm, float* dS,
                              ConvGeom g) {
    const int K = g.C * g.k * g.k;
    const int64_t total = static_cast<int64_t>(g.N) * g.C * g.H * g.W;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int w = static_cast<int>(i % g.W);
        const int h = static_cast<int>((i / g.W) % g.H);
        const int c = static_cast<int>((i / (static_cast<int64_t>(g.W) * g.H)) % g.C);
        const int n = static_cast<int>(i / (static_cast<int64_t>(g.W) * g.H * g.C));
        float am = 0.f, aS = 0.f;
        for (int kh = 0; kh < g.k; ++kh) {
            const int ohn = h + g.p_tl - kh;
            // C division truncates toward zero, matching Triton's integer
            // semantics in the reference kernel (conv2d.py:122-126).
            const int oh = ohn / g.s;
            const bool okh = (ohn % g.s == 0) && oh >= 0 && oh < g.Ho && (!ADJOINT || ohn >= 0);
            for (int kw = 0; kw < g.k; ++kw) {
                const int own = w + g.p_tl - kw;
                const int ow = own / g.s;
                // The reference accepts a tap without testing own % stride
                // (conv2d.py:126); the adjoint requires it.
                const bool okw = ow >= 0 && ow < g.Wo && (!ADJOINT || (own >= 0 && own % g.s == 0));
                if (okh && okw) {
                    const int64_t src =
                        ((static_cast<int64_t>(n) * g.Ho + oh) * g.Wo + ow) * K +
                        (c * g.k + kh) * g.k + kw;
                    am += cm[src];
                    aS += cS[src];
                }
            }
        }
        dm[i] = am;
        dS[i] = aS;
    }
}

// The same gather per (image, channel slice) CTA: the patch columns of the
// slice for all L = Ho*Wo patch rows of the image (both planes) are staged in
// shared memory with coalesced asynchronous copies (each row contributes cs*k*k
// contiguous floats), then each thread gathers output pixels (c, h, w) from
// shared memory, visiting taps in the same (kh, kw) order, so the sums are
// bit-identical to col2im_kernel.
// q / S and q % S with C semantics (truncation toward zero); S = 0 reads the
// stride at run time, S = 2 uses shifts.
template <int S>
__device__ __forceinline__ void div_trunc(int q, int s, int* quo, bool* exact) {
    if (S == 2) {
        *quo = q >= 0 ? (q >> 1) : -((-q) >> 1);
        *exact = (q & 1) == 0;
    } else {
        *quo = q / s;
        *exact = q % s == 0;
    }
}

template <bool ADJOINT, int S>
__global__ void col2im_img_kernel(const float* cm, const float* cS, float* dm, float* dS,
                                  ConvGeom g, int cslice) {
    extern __shared__ float patch[];  // [plane][L][rs]
    const int kk = g.k * g.k, K = g.C * kk, L = g.Ho * g.Wo;
    const int nslice = (g.C + cslice - 1) / cslice;
    const int n = blockIdx.x / nslice, c0 = (blockIdx.x - n * nslice) * cslice;
    const int cs = min(cslice, g.C - c0);
    const int q = cs * kk, rs = (cslice * kk) | 1;  // columns staged per row; odd row stride
    const int tid = threadIdx.x, nth = blockDim.x;
    const float rq = 1.f / q;
    const int64_t base = static_cast<int64_t>(n) * L * K + static_cast<int64_t>(c0) * kk;
    for (int e = tid; e < L * q; e += nth) {
        const int r = div_small(e, rq), j = e - r * q;
        const int64_t src = base + static_cast<int64_t>(r) * K + j;
        cp_async4(patch + r * rs + j, cm + src, true);
        cp_async4(patch + (L + r) * rs + j, cS + src, true);
    }
    cp_async_wait_all();
    __syncthreads();
    const int hw = g.H * g.W, total = cs * hw;
    const float rW = 1.f / g.W, rhw = 1.f / hw;
    for (int i = tid; i < total; i += nth) {
        const int cl = div_small(i, rhw), p = i - cl * hw;
        const int h = div_small(p, rW), w = p - h * g.W;
        float am = 0.f, aS = 0.f;
        for (int kh = 0; kh < g.k; ++kh) {
            int oh;
            bool exh;
            div_trunc<S>(h + g.p_tl - kh, g.s, &oh, &exh);  // truncates toward zero, as the reference
            const bool okh = exh && oh >= 0 && oh < g.Ho && (!ADJOINT || h + g.p_tl - kh >= 0);
            if (!okh) continue;
            for (int kw = 0; kw < g.k; ++kw) {
                const int own = w + g.p_tl - kw;
                int ow;
                bool exw;
                div_trunc<S>(own, g.s, &ow, &exw);
                const bool okw = ow >= 0 && ow < g.Wo && (!ADJOINT || (own >= 0 && exw));
                if (okw) {
                    const int o = (oh * g.Wo + ow) * rs + cl * kk + kh * g.k + kw;
                    am += patch[o];
                    aS += patch[L * rs + o];
                }
            }
        }
        const int64_t out = (static_cast<int64_t>(n) * g.C + c0 + cl) * hw + p;
        dm[out] = am;
        dS[out] = aS;
    }
}

// 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// Stride-2 gather with the kernel size known at compile time (KS = 2 or 3),
// one CTA per (image, slice of cs channels): the slice's patch columns (cs*k*k
// contiguous floats of each of the L patch rows, both planes) are staged with
// 16-byte asynchronous copies (row stride rs = 4 mod 8 floats: a warp's reads
// hit at most two rows per bank); then each thread sums 4 consecutive input
// pixels of one row of one channel and stores them with one 16-byte store. A
// warp covers one input row h of 32 / (W / 4) channels, so the taps kh that
// reach the row are the same for the whole warp. Each pixel visits its taps in
// (kh, kw) order, as col2im_kernel does, so the sums are bit-identical to it.
template <int KS, bool ADJOINT>
__global__ void __launch_bounds__(256) col2im_s2_kernel(const float* cm, const float* cS,
                                                        float* dm, float* dS, ConvGeom g, int cs,
                                                        int rs) {
    extern __shared__ __align__(16) float stage[];  // [plane][L][rs]
    constexpr int KK = KS * KS;
    const int K = g.C * KK, L = g.Ho * g.Wo;
    const int nslice = g.C / cs;
    const int n = blockIdx.x / nslice, c0 = (blockIdx.x - n * nslice) * cs;
    const int q4 = cs * KK / 4;  // 16-byte chunks of a patch row
    const float rq4 = 1.f / q4;
    const int64_t base = static_cast<int64_t>(n) * L * K + static_cast<int64_t>(c0) * KK;
    for (int e = threadIdx.x; e < L * q4; e += blockDim.x) {
        const int r = div_small(e, rq4), j = e - r * q4;
        const int64_t src = base + static_cast<int64_t>(r) * K + 4 * j;
        cp_async16(stage + r * rs + 4 * j, cm + src);
        cp_async16(stage + (L + r) * rs + 4 * j, cS + src);
    }
    cp_async_wait_all();
    __syncthreads();
    const int W4 = g.W >> 2, units = cs * g.H * W4;
    const float rW4 = 1.f / W4, rcs = 1.f / cs;
    const int64_t plane = static_cast<int64_t>(g.H) * g.W;
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
        const int t = div_small(u, rW4), wg = u - t * W4;
        const int h = div_small(t, rcs), cl = t - h * cs;
        float am[4] = {0.f, 0.f, 0.f, 0.f}, aS[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kh = 0; kh < KS; ++kh) {
            const int ohn = h + g.p_tl - kh;
            // the reference's test (ohn % 2 == 0 with truncating division):
            // odd numerators, negative ones included, never contribute
            if (ohn & 1) continue;
            const int oh = ohn / 2;
            if (oh < 0 || oh >= g.Ho) continue;
            const float* prow = stage + oh * g.Wo * rs + cl * KK + kh * KS;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int w = 4 * wg + e;
#pragma unroll
                for (int kw = 0; kw < KS; ++kw) {
                    const int own = w + g.p_tl - kw;
                    const int ow = own >= 0 ? (own >> 1) : -((-own) >> 1);  // truncating
                    // the reference does not test own % 2 (conv2d.py:126); the adjoint does
                    const bool ok = ow >= 0 && ow < g.Wo && (!ADJOINT || (own >= 0 && !(own & 1)));
                    if (ok) {
                        am[e] += prow[ow * rs + kw];
                        aS[e] += prow[(L + ow) * rs + kw];
                    }
                }
            }
        }
        const int64_t o = (static_cast<int64_t>(n) * g.C + c0 + cl) * plane +
                          static_cast<int64_t>(h) * g.W + 4 * wg;
        *reinterpret_cast<float4*>(dm + o) = make_float4(am[0], am[1], am[2], am[3]);
        *reinterpret_cast<float4*>(dS + o) = make_float4(aS[0], aS[1], aS[2], aS[3]);
    }
}

// Channel slice and shared row stride of col2im_s2_kernel (cs = 0: not
// applicable): the largest power-of-two slice dividing C whose staging fits
// 76 KB (three CTAs per SM), rows padded to 4 mod 8 floats.
inline void col2im_s2_plan(const ConvGeom& g, int* cs_out, int* rs_out) {
    *cs_out = 0;
    const int kk = g.k * g.k, L = g.Ho * g.Wo;
    if (g.s != 2 || (g.k != 2 && g.k != 3) || g.W % 4 != 0 || g.C % 4 != 0) return;
    for (int cs = 1; cs <= g.C && cs <= 1024; cs *= 2) {
        if (g.C % cs || (cs * kk) % 4) continue;
        const int rs = (cs * kk) % 8 == 0 ? cs * kk + 4 : cs * kk;
        if (2ll * L * rs * 4 > 76 * 1024) break;
        *cs_out = cs;
        *rs_out = rs;
    }
}

// 16-byte asynchronous copy global -> shared, zero-filled when !ok (the
// source is then not read).
__device__ __forceinline__ void cp_async16_zfill(float* dst, const float* src, bool ok) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
                 "r"(ok ? 16 : 0)
                 : "memory");
}

// Patches of one output image row (image n, output row oh) per CTA with the
// kernel size known at compile time (KS = 2 or 3) and every channel staged at
// once: the C*KS input lines (oh*s - p + kh, W columns each; zeros for lines
// outside the image) arrive by 16-byte asynchronous copies (line stride W + 4
// floats), then each thread owns patch columns and walks the row's pixels
// (index decoding once per column; a warp stores 32 consecutive columns of one
// patch row per step). Needs W and K = C*KS*KS multiples of 4 and 16-byte
// aligned pointers.
template <int KS, int PLANES>
__global__ void __launch_bounds__(256) im2col_row4_kernel(const float* xm, const float* xS,
                                                          float* pm, float* pS, ConvGeom g) {
    extern __shared__ __align__(16) float lines[];  // [plane][C * KS lines][W + 4]
    constexpr int KK = KS * KS;
    const int ls = g.W + 4, W4 = g.W >> 2;
    const int n = blockIdx.x / g.Ho, oh = blockIdx.x - n * g.Ho;
    const int K = g.C * KK, nlines = g.C * KS, pstride = nlines * ls;
    const int ih0 = oh * g.s - g.p_tl;
    const int64_t img = static_cast<int64_t>(n) * g.C * g.H * g.W;
    const float rW4 = 1.f / W4;
    for (int e = threadIdx.x; e < PLANES * nlines * W4; e += blockDim.x) {
        int li = div_small(e, rW4);
        const int q = e - li * W4;
        const int pl = (PLANES == 2 && li >= nlines) ? 1 : 0;
        li -= pl * nlines;
        const int c = li / KS, ih = ih0 + (li - c * KS);
        const bool in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
        const float* src =
            (pl ? xS : xm) + img + (static_cast<int64_t>(c) * g.H + (in ? ih : 0)) * g.W + 4 * q;
        cp_async16_zfill(lines + pl * pstride + li * ls + 4 * q, src, in);
    }
    cp_async_wait_all();
    __syncthreads();
    // thread t owns patch columns j = t, t + blockDim.x, ... and walks the row's
    // Wo pixels: a warp stores 32 consecutive columns of one patch row per step
    const int64_t out0 = static_cast<int64_t>(blockIdx.x) * g.Wo * K;  // patch row (n, oh, 0)
    for (int j = threadIdx.x; j < K; j += blockDim.x) {
        const int c = j / KK, t = j - c * KK;
        const int kh = t / KS, kw = t - kh * KS;
        const float* line = lines + (c * KS + kh) * ls;
        float* om = pm + out0 + j;
        float* oS = PLANES == 2 ? pS + out0 + j : nullptr;
        int iw = kw - g.p_tl;
#pragma unroll 4
        for (int ow = 0; ow < g.Wo; ++ow, iw += g.s, om += K) {
            const bool in = static_cast<unsigned>(iw) < static_cast<unsigned>(g.W);
            const int a = in ? iw : 0;
            *om = in ? line[a] : 0.f;
            if (PLANES == 2) {
                *oS = in ? line[pstride + a] : 0.f;
                oS += K;
            }
        }
    }
}

// NCHW -> NHWC of one or two planes over the flattened pixel index q = n*HW + p:
// 32 x 32 tiles of (channel, q) through shared memory (padded against bank
// conflicts). Reads run along q (contiguous within each image plane, so small
// maps still fill whole tiles), writes along the channels of one pixel.
__global__ void nchw_to_nhwc_kernel(const float* xm, const float* xS, float* ym, float* yS,
                                    int C, int HW, int64_t Q) {
    __shared__ float tile[2][32][33];
    const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int c0 = blockIdx.y * 32;
    {
        const int64_t q = q0 + threadIdx.x;
        const int64_t n = q / HW, p = q - n * HW;
        for (int r = threadIdx.y; r < 32; r += blockDim.y) {
            const int c = c0 + r;
            if (c < C && q < Q) {
                const int64_t src = (n * C + c) * HW + p;
                tile[0][r][threadIdx.x] = xm[src];
                if (xS) tile[1][r][threadIdx.x] = xS[src];
            }
        }
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int64_t q = q0 + r;
        const int c = c0 + threadIdx.x;
        if (c < C && q < Q) {
            ym[q * C + c] = tile[0][threadIdx.x][r];
            if (xS) yS[q * C + c] = tile[1][threadIdx.x][r];
        }
    }
}

// The same copy with 128-bit accesses when HW and C are multiples of 4 (and
// the tensors 16-byte aligned, Q < 2^31): tiles of 32 channels x 64 pixels;
// each thread loads 4 consecutive pixels of one channel and stores 4
// consecutive channels of one pixel. Row pitch 65 keeps both shared-memory
// phases free of bank conflicts beyond 2-way.
__global__ void __launch_bounds__(256) nchw_to_nhwc_v4_kernel(const float* xm, const float* xS,
                                                              float* ym, float* yS, int C, int HW,
                                                              int Q) {
    __shared__ float tile[2][32][65];
    const int q0 = blockIdx.x * 64, c0 = blockIdx.y * 32;
    const int planes = xS ? 2 : 1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int idx = threadIdx.x + 256 * j, c = idx >> 4, q4 = idx & 15;
        const int q = q0 + 4 * q4;
        if (q < Q && c0 + c < C) {
            const int n = q / HW, p = q - n * HW;
            const int64_t src = (static_cast<int64_t>(n) * C + c0 + c) * HW + p;
            for (int pl = 0; pl < planes; ++pl) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>((pl ? xS : xm) + src));
                float* t = &tile[pl][c][4 * q4];
                t[0] = v.x; t[1] = v.y; t[2] = v.z; t[3] = v.w;
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int idx = threadIdx.x + 256 * j, ql = idx >> 3, cg = idx & 7;
        const int q = q0 + ql, c = c0 + 4 * cg;
        if (q < Q && c < C) {
            const int64_t dst = static_cast<int64_t>(q) * C + c;
            for (int pl = 0; pl < planes; ++pl) {
                const float4 v = make_float4(tile[pl][4 * cg][ql], tile[pl][4 * cg + 1][ql],
                                             tile[pl][4 * cg + 2][ql], tile[pl][4 * cg + 3][ql]);
                *reinterpret_cast<float4*>((pl ? yS : ym) + dst) = v;
            }
        }
    }
}

// Transposed mean patches: row i = (c, kh, kw) of PT holds, for every output
// pixel q = (n, oh, ow), x[n][c][oh*s - p + kh][ow*s - p + kw] (0 outside the
// image). One CTA per (n, c, band of TH output rows): the band's input rows
// ((TH-1)*s + k of them, one contiguous range of the plane; rows outside the
// image staged as zeros) go to shared memory, then each of the k*k patch rows
// of the band is written as one contiguous run of TH*Wo pixels, four per thread
// and 128-bit store when V4 (Wo and Q multiples of 4).
template <bool V4>
__global__ void __launch_bounds__(256) im2col_t_band_kernel(const float* x, float* pt, ConvGeom g,
                                                            int64_t Q, int TH, int bands) {
    extern __shared__ float sx[];
    const int band = static_cast<int>(blockIdx.x % bands);
    const int64_t nc = blockIdx.x / bands;
    const int n = static_cast<int>(nc / g.C), c = static_cast<int>(nc - static_cast<int64_t>(n) * g.C);
    const int oh0 = band * TH, th = min(TH, g.Ho - oh0);
    const int rows_in = (th - 1) * g.s + g.k;
    const int64_t plane_len = static_cast<int64_t>(g.H) * g.W;
    const float* plane = x + nc * plane_len;
    const int64_t first = static_cast<int64_t>(oh0 * g.s - g.p_tl) * g.W;  // may be negative
    const int staged = rows_in * g.W;
    for (int i = threadIdx.x; i < staged; i += blockDim.x) {
        const int64_t o = first + i;
        sx[i] = (o >= 0 && o < plane_len) ? __ldg(plane + o) : 0.f;
    }
    __syncthreads();
    const int cnt = th * g.Wo, kk = g.k * g.k;
    const float rWo = 1.f / g.Wo;
    const int64_t col0 = static_cast<int64_t>(n) * g.Ho * g.Wo + static_cast<int64_t>(oh0) * g.Wo;
    for (int t = 0; t < kk; ++t) {
        const int kh = t / g.k, kw = t - kh * g.k;
        float* out = pt + (static_cast<int64_t>(c) * kk + t) * Q + col0;
        if (V4) {
            for (int j = 4 * threadIdx.x; j < cnt; j += 4 * blockDim.x) {
                const int ol = div_small(j, rWo), ow = j - ol * g.Wo;  // 4 pixels of one row
                const float* row = sx + (ol * g.s + kh) * g.W;
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int iw = (ow + e) * g.s - g.p_tl + kw;
                    v[e] = static_cast<unsigned>(iw) < static_cast<unsigned>(g.W) ? row[iw] : 0.f;
                }
                *reinterpret_cast<float4*>(out + j) = make_float4(v[0], v[1], v[2], v[3]);
            }
        } else {
            for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
                const int ol = div_small(j, rWo), ow = j - ol * g.Wo;
                const int iw = ow * g.s - g.p_tl + kw;
                out[j] = static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)
                             ? sx[(ol * g.s + kh) * g.W + iw]
                             : 0.f;
            }
        }
    }
}

// Stride-1 transposed patches for k = K <= 5 with Wo a multiple of 4: the band's
// input rows are staged zero-padded (padded column x = input column + p_tl, row
// pitch Wo + 4), so that the K taps of a row, for 4 consecutive output pixels
// ow..ow+3, are padded columns ow+kw .. ow+kw+3: two aligned 128-bit shared
// loads (columns ow..ow+7) serve all K taps of one kernel row, without bounds
// tests, and each tap leaves as one 128-bit store.
template <int K>
__global__ void __launch_bounds__(256) im2col_t_s1_kernel(const float* x, float* pt, ConvGeom g,
                                                          int64_t Q, int TH, int bands) {
    extern __shared__ __align__(16) float sx1[];
    const int band = static_cast<int>(blockIdx.x % bands);
    const int64_t nc = blockIdx.x / bands;
    const int n = static_cast<int>(nc / g.C), c = static_cast<int>(nc - static_cast<int64_t>(n) * g.C);
    const int oh0 = band * TH, th = min(TH, g.Ho - oh0);
    const int rows_in = th + K - 1, Wp = g.Wo + 4;
    const float* plane = x + nc * static_cast<int64_t>(g.H) * g.W;
    const float rWp = 1.f / Wp;
    for (int i = threadIdx.x; i < rows_in * Wp; i += blockDim.x) {
        const int r = div_small(i, rWp), xc = i - r * Wp;
        const int ih = oh0 - g.p_tl + r, iw = xc - g.p_tl;
        sx1[i] = (static_cast<unsigned>(ih) < static_cast<unsigned>(g.H) &&
                 static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
                    ? __ldg(plane + static_cast<int64_t>(ih) * g.W + iw)
                    : 0.f;
    }
    __syncthreads();
    const int cnt = th * g.Wo;
    const float rWo = 1.f / g.Wo;
    float* base = pt + static_cast<int64_t>(c) * K * K * Q + static_cast<int64_t>(n) * g.Ho * g.Wo +
                  static_cast<int64_t>(oh0) * g.Wo;
    for (int j = 4 * threadIdx.x; j < cnt; j += 4 * blockDim.x) {
        const int ol = div_small(j, rWo), ow = j - ol * g.Wo;
        float* o = base + j;
#pragma unroll
        for (int kh = 0; kh < K; ++kh) {
            const float* row = sx1 + (ol + kh) * Wp + ow;
            const float4 a = *reinterpret_cast<const float4*>(row);
            const float4 b = *reinterpret_cast<const float4*>(row + 4);
            const float w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int kw = 0; kw < K; ++kw) {
                *reinterpret_cast<float4*>(o) = make_float4(w[kw], w[kw + 1], w[kw + 2], w[kw + 3]);
                o += Q;
            }
        }
    }
}

// The same patches one element per thread, for images too wide to stage k rows
// (grid row = patch row i).
__global__ void im2col_t_kernel(const float* x, float* pt, ConvGeom g, int64_t Q) {
    const int i = blockIdx.y;
    const int kk = g.k * g.k, c = i / kk, t = i - c * kk, kh = t / g.k, kw = t - kh * g.k;
    const int64_t L = static_cast<int64_t>(g.Ho) * g.Wo;
    float* out = pt + static_cast<int64_t>(i) * Q;
    const int64_t plane = static_cast<int64_t>(g.H) * g.W;
    for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < Q;
         q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = q / L;
        const int l = static_cast<int>(q - n * L), oh = l / g.Wo, ow = l - oh * g.Wo;
        const int ih = oh * g.s - g.p_tl + kh, iw = ow * g.s - g.p_tl + kw;
        const bool in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H) &&
                        static_cast<unsigned>(iw) < static_cast<unsigned>(g.W);
        out[q] = in ? __ldg(x + (n * g.C + c) * plane + static_cast<int64_t>(ih) * g.W + iw) : 0.f;
    }
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" int tagi_im2col(const float* xm, const float* xS, float* pm, float* pS, int64_t N,
                           int64_t C, int64_t H, int64_t W, int64_t k, int64_t stride,
                           int64_t padding, int64_t padding_type, void* stream) {
    const char* what = "tagi_im2col";
    ConvGeom g;
    TAGI_REQUIRE(make_geom(N, C, H, W, k, stride, padding, padding_type, &g), TAGI_E_BAD_ARG,
                 "%s: bad geometry", what);
    const int64_t total = N * g.Ho * g.Wo * C * k * k;
    if (total == 0) return TAGI_OK;
    TAGI_REQUIRE(xm && pm && (xS == nullptr) == (pS == nullptr), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    {
        // every channel's lines staged at once, 16-byte copies and stores
        const int64_t smem = (xS ? 2 : 1) * C * k * (W + 4) * static_cast<int64_t>(sizeof(float));
        const uintptr_t a16 = reinterpret_cast<uintptr_t>(xm) | reinterpret_cast<uintptr_t>(xS) |
                              reinterpret_cast<uintptr_t>(pm) | reinterpret_cast<uintptr_t>(pS);
        if ((k == 2 || k == 3) && W % 4 == 0 && (C * k * k) % 4 == 0 && (a16 & 15) == 0 &&
            smem <= 96 * 1024 && N * g.Ho <= INT_MAX &&
            static_cast<int64_t>(g.Wo) * C * k * k < (int64_t(1) << 22)) {
            static bool attr_set[4] = {false, false, false, false};
            const unsigned grid = static_cast<unsigned>(N * g.Ho);
            cudaStream_t st = as_stream(stream);
            auto run = [&](auto kernel, int which) {
                if (!attr_set[which]) {
                    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         96 * 1024);
                    attr_set[which] = true;
                }
                kernel<<<grid, 256, static_cast<size_t>(smem), st>>>(xm, xS, pm, pS, g);
            };
            if (k == 3)
                xS ? run(im2col_row4_kernel<3, 2>, 0) : run(im2col_row4_kernel<3, 1>, 1);
            else
                xS ? run(im2col_row4_kernel<2, 2>, 2) : run(im2col_row4_kernel<2, 1>, 3);
            return check_launch(what);
        }
    }
    // staged lines of a channel slice within 32 KB of shared memory
    const int64_t line_bytes = (xS ? 2 : 1) * k * (W | 1) * static_cast<int64_t>(sizeof(float));
    const int64_t cslice = std::min<int64_t>(C, (32 * 1024) / line_bytes);
    const uintptr_t al = (reinterpret_cast<uintptr_t>(pm) | reinterpret_cast<uintptr_t>(pS)) & 15;
    // div_small bounds: staged elements (<= 8192) and patch columns below 2^22
    if (cslice >= 1 && N * g.Ho <= INT_MAX && C * k * k < (int64_t(1) << 22)) {
        const unsigned grid = static_cast<unsigned>(N * g.Ho);
        const size_t smem = static_cast<size_t>(cslice * line_bytes);
        if (xS)
            im2col_rows_kernel<2><<<grid, 256, smem, as_stream(stream)>>>(
                xm, xS, pm, pS, g, static_cast<int>(cslice));
        else
            im2col_rows_kernel<1><<<grid, 256, smem, as_stream(stream)>>>(
                xm, xS, pm, pS, g, static_cast<int>(cslice));
    } else if ((C * k * k) % 4 == 0 && al == 0) {
        im2col_v4_kernel<<<grid_1d(total / 4, 256), 256, 0, as_stream(stream)>>>(xm, xS, pm, pS, g);
    } else {
        im2col_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(xm, xS, pm, pS, g);
    }
    return check_launch(what);
}

extern "C" int tagi_col2im(const float* cm, const float* cS, float* dm, float* dS, int64_t N,
                           int64_t C, int64_t H, int64_t W, int64_t k, int64_t stride,
                           int64_t padding, int64_t padding_type, int mode, void* stream) {
    const char* what = "tagi_col2im";
    ConvGeom g;
    TAGI_REQUIRE(make_geom(N, C, H, W, k, stride, padding, padding_type, &g), TAGI_E_BAD_ARG,
                 "%s: bad geometry", what);
    TAGI_REQUIRE(mode == 0 || mode == 1, TAGI_E_BAD_ARG, "%s: mode must be 0 or 1", what);
    const int64_t total = N * C * H * W;
    if (total == 0) return TAGI_OK;
    TAGI_REQUIRE(cm && cS && dm && dS, TAGI_E_BAD_ARG, "%s: null pointer", what);
    {
        int cs = 0, rs = 0;
        col2im_s2_plan(g, &cs, &rs);
        const uintptr_t al = reinterpret_cast<uintptr_t>(cm) | reinterpret_cast<uintptr_t>(cS) |
                             reinterpret_cast<uintptr_t>(dm) | reinterpret_cast<uintptr_t>(dS);
        const int64_t ctas = cs > 0 ? N * (C / cs) : 0;
        if (cs > 0 && (al & 15) == 0 && ctas <= INT_MAX &&
            static_cast<int64_t>(g.Ho) * g.Wo * C * k * k < (int64_t(1) << 22)) {
            static bool attr_set[4] = {false, false, false, false};
            const size_t smem = 2ull * g.Ho * g.Wo * rs * sizeof(float);
            cudaStream_t st = as_stream(stream);
            auto run = [&](auto kernel, int which) {
                if (!attr_set[which]) {
                    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         76 * 1024);
                    attr_set[which] = true;
                }
                kernel<<<static_cast<unsigned>(ctas), 256, smem, st>>>(cm, cS, dm, dS, g, cs, rs);
            };
            if (k == 3)
                mode == 0 ? run(col2im_s2_kernel<3, false>, 0) : run(col2im_s2_kernel<3, true>, 1);
            else
                mode == 0 ? run(col2im_s2_kernel<2, false>, 2) : run(col2im_s2_kernel<2, true>, 3);
            return check_launch(what);
        }
    }
    // Staged per (image, channel slice) when one channel's patch columns for the
    // image fit: both planes of L rows x cslice*k*k columns within 48 KB.
    const int64_t L = static_cast<int64_t>(g.Ho) * g.Wo, kk = k * k;
    const int64_t per_c = 2 * L * kk * static_cast<int64_t>(sizeof(float));
    const int64_t budget = 48 * 1024;  // 4 CTAs per SM: staging overlaps gathering
    int64_t cslice = per_c > 0 ? std::min<int64_t>(C, budget / per_c) : 0;
    // the odd row stride may add one column per row
    while (cslice >= 1 && 2 * L * ((cslice * kk) | 1) * 4 > budget) --cslice;
    const int64_t ctas = cslice >= 1 ? N * ((C + cslice - 1) / cslice) : 0;
    const bool small = L * C * kk < (int64_t(1) << 22) && H * W * cslice < (int64_t(1) << 22);
    if (cslice >= 1 && ctas <= INT_MAX && small) {
        static bool attr_set[4] = {false, false, false, false};
        const size_t smem = static_cast<size_t>(2 * L * ((cslice * kk) | 1) * 4);
        cudaStream_t st = as_stream(stream);
        auto run = [&](auto kernel, int which) {
            if (!attr_set[which]) {
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
                attr_set[which] = true;
            }
            kernel<<<static_cast<unsigned>(ctas), 256, smem, st>>>(cm, cS, dm, dS, g,
                                                                  static_cast<int>(cslice));
        };
        if (mode == 0)
            stride == 2 ? run(col2im_img_kernel<false, 2>, 0) : run(col2im_img_kernel<false, 0>, 1);
        else
            stride == 2 ? run(col2im_img_kernel<true, 2>, 2) : run(col2im_img_kernel<true, 0>, 3);
    } else if (mode == 0) {
        col2im_kernel<false><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(cm, cS, dm, dS, g);
    } else {
        col2im_kernel<true><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(cm, cS, dm, dS, g);
    }
    return check_launch(what);
}

extern "C" int tagi_nchw_to_nhwc(const float* xm, const float* xS, float* ym, float* yS, int64_t N,
                                 int64_t C, int64_t HW, void* stream) {
    const char* what = "tagi_nchw_to_nhwc";
    TAGI_REQUIRE(N >= 0 && C >= 0 && HW >= 0 && C <= 65535 * 32 &&
                     N * C * HW < (int64_t(1) << 40),
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (N == 0 || C == 0 || HW == 0) return TAGI_OK;
    TAGI_REQUIRE(xm && ym && (xS == nullptr) == (yS == nullptr), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    const int64_t Q = N * HW;
    TAGI_REQUIRE((Q + 31) / 32 <= INT_MAX, TAGI_E_BAD_ARG, "%s: too many pixels", what);
    const uintptr_t al = (reinterpret_cast<uintptr_t>(xm) | reinterpret_cast<uintptr_t>(xS) |
                          reinterpret_cast<uintptr_t>(ym) | reinterpret_cast<uintptr_t>(yS)) & 15;
    if (HW % 4 == 0 && C % 4 == 0 && al == 0 && Q < INT_MAX) {
        const dim3 grid(static_cast<unsigned>((Q + 63) / 64), static_cast<unsigned>((C + 31) / 32), 1);
        nchw_to_nhwc_v4_kernel<<<grid, 256, 0, as_stream(stream)>>>(xm, xS, ym, yS, (int)C,
                                                                    (int)HW, (int)Q);
        return check_launch(what);
    }
    const dim3 grid(static_cast<unsigned>((Q + 31) / 32), static_cast<unsigned>((C + 31) / 32), 1);
    nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(xm, xS, ym, yS, (int)C,
                                                                       (int)HW, Q);
    return check_launch(what);
}

extern "C" int tagi_im2col_t(const float* x, float* pt, int64_t N, int64_t C, int64_t H,
                             int64_t W, int64_t k, int64_t stride, int64_t padding,
                             int64_t padding_type, void* stream) {
    const char* what = "tagi_im2col_t";
    ConvGeom g;
    TAGI_REQUIRE(make_geom(N, C, H, W, k, stride, padding, padding_type, &g), TAGI_E_BAD_ARG,
                 "%s: bad geometry", what);
    const int64_t Q = N * g.Ho * g.Wo, rows = C * k * k;
    if (Q == 0 || rows == 0) return TAGI_OK;
    TAGI_REQUIRE(x && pt, TAGI_E_BAD_ARG, "%s: null pointer", what);
    // band kernel: staged rows within 24 KB, band pixels (div_small) below 2^22
    constexpr int64_t kStage = 24 * 1024 / sizeof(float);
    const bool al16 = (reinterpret_cast<uintptr_t>(pt) & 15) == 0;
    const int64_t rows_s1 = kStage / (g.Wo + 4);
    if (stride == 1 && (k == 1 || k == 3 || k == 5) && g.Wo % 4 == 0 && Q % 4 == 0 && al16 &&
        rows_s1 >= k) {
        const int64_t TH = std::min<int64_t>({static_cast<int64_t>(g.Ho), rows_s1 - k + 1,
                                              ((int64_t(1) << 22) - 1) / g.Wo});
        const int64_t bands = (g.Ho + TH - 1) / TH;
        const size_t smem = static_cast<size_t>((TH + k - 1) * (g.Wo + 4)) * sizeof(float);
        const int64_t blocks = N * C * bands;
        TAGI_REQUIRE(blocks <= INT_MAX, TAGI_E_UNSUPPORTED, "%s: too many planes", what);
        const unsigned nb = static_cast<unsigned>(blocks);
        const int th = static_cast<int>(TH), nbands = static_cast<int>(bands);
        if (k == 1)
            im2col_t_s1_kernel<1><<<nb, 256, smem, as_stream(stream)>>>(x, pt, g, Q, th, nbands);
        else if (k == 3)
            im2col_t_s1_kernel<3><<<nb, 256, smem, as_stream(stream)>>>(x, pt, g, Q, th, nbands);
        else
            im2col_t_s1_kernel<5><<<nb, 256, smem, as_stream(stream)>>>(x, pt, g, Q, th, nbands);
        return check_launch(what);
    }
    const int64_t rows_max = kStage / W;
    if (rows_max >= k) {
        const int64_t TH = std::min<int64_t>({static_cast<int64_t>(g.Ho), (rows_max - k) / stride + 1,
                                              ((int64_t(1) << 22) - 1) / g.Wo});
        const int64_t bands = (g.Ho + TH - 1) / TH;
        const size_t smem = static_cast<size_t>(((TH - 1) * stride + k) * W) * sizeof(float);
        const bool v4 = g.Wo % 4 == 0 && Q % 4 == 0 && (reinterpret_cast<uintptr_t>(pt) & 15) == 0;
        const int64_t blocks = N * C * bands;
        TAGI_REQUIRE(blocks <= INT_MAX, TAGI_E_UNSUPPORTED, "%s: too many planes", what);
        if (v4)
            im2col_t_band_kernel<true><<<static_cast<unsigned>(blocks), 256, smem, as_stream(stream)>>>(
                x, pt, g, Q, static_cast<int>(TH), static_cast<int>(bands));
        else
            im2col_t_band_kernel<false><<<static_cast<unsigned>(blocks), 256, smem, as_stream(stream)>>>(
                x, pt, g, Q, static_cast<int>(TH), static_cast<int>(bands));
        return check_launch(what);
    }
    TAGI_REQUIRE(rows <= 65535, TAGI_E_UNSUPPORTED, "%s: too many patch rows", what);
    const unsigned bx = static_cast<unsigned>(std::min<int64_t>((Q + 255) / 256, 4096));
    im2col_t_kernel<<<dim3(bx, static_cast<unsigned>(rows)), 256, 0, as_stream(stream)>>>(x, pt, g, Q);
    return check_launch(what);
}
