// Patch extraction and patch-delta gathering for the im2col Conv2D path.
//
// Layout follows the reference: patches are (N*Ho*Wo) x (C*k*k) row-major with
// row = (n, oh, ow) and column = (c, kh, kw); images are NCHW.
// padding_type 2 pads only the right/bottom edge by `padding`
// (triton_tagi/layers/conv2d.py:280-291), i.e. the top-left offset is 0.
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
    const uintptr_t al = (reinterpret_cast<uintptr_t>(pm) | reinterpret_cast<uintptr_t>(pS)) & 15;
    if ((C * k * k) % 4 == 0 && al == 0) {
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
    if (mode == 0)
        col2im_kernel<false><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(cm, cS, dm, dS, g);
    else
        col2im_kernel<true><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(cm, cS, dm, dS, g);
    return check_launch(what);
}
