// Shared definitions of the moment-contraction kernels (CUDA-core and tcgen05).
#pragma once

#include "common.cuh"

namespace tagi {

enum VarMode { FULL = 0, RSQ = 1, LSQ = 2 };
enum Epi { EPI_STORE = 0, EPI_PARTIAL = 1, EPI_PARAM = 2 };

struct ParamEpi {
    int mode;  // TAGI_WGRAD_SUMS / DELTAS / UPDATE
    int K, N;  // weight rows, columns; row K is the bias row when present
    float *mw, *Sw, *mb, *Sb;
    float *out_m, *out_S, *out_mb, *out_Sb;
    float cap;
};

// Implicit patches on the A side (convolutions without a patch matrix). Rows
// m = (n, y, x) run over an N x (L/Wo) x Wo pixel grid, the reduction index is
// r = tap*C + c with tap = kh*k + kw (taps outermost: 8 consecutive reduction
// elements then share one tap for C a multiple of 8, i.e. one bounds test and
// 8 addresses a channel plane apart). The B operand is read in the same order.
//   mode 0, patches (Conv2D forward): A[m][r] = x[n][c][y*s - pt + kh][x*s - pl + kw]
//     (triton_tagi/layers/conv2d.py:40-77), zero outside the input;
//   mode 1, the reference's col2im gather (conv2d.py:119-130) of the deltas of a
//     C x H x W output onto input pixel (y, x): tap (kh, kw) contributes
//     x[n][c][oh][ow] with ohn = y + pt - kh, own = x + pl - kw, oh = ohn / s and
//     ow = own / s truncating toward zero, if ohn % s == 0, 0 <= oh < H and
//     0 <= ow < W (the column offset is not tested for divisibility);
//   mode 2, the adjoint of the patches: mode 1 plus ohn, own >= 0 and own % s == 0.
// nhwc: the gathered tensor is channels-last (N x H x W x C), so the 8 channels
// of a reduction block at one tap are 32 contiguous bytes (one 256-bit load
// when C is a multiple of 8) instead of 8 values a channel plane apart.
struct Gather {
    int on;              // 1: A is gathered; arow and ak are unused
    int mode;            // 0 patches, 1 reference col2im gather, 2 adjoint gather
    int C, H, W;         // gathered tensor's channels and size
    int Wo, L;           // row pixel grid: width, pixels per image
    int k, s, pt, pl;    // kernel size, stride, top and left padding
    int nhwc;            // 0: NCHW, 1: NHWC
};

// One row pixel's image base and origin: mode 0, the input position of tap
// (0, 0); modes 1-2, (y + pt, x + pl).
struct GatherRow {
    int64_t base;
    int ih0, iw0;
};

__device__ __forceinline__ GatherRow gather_row(const Gather& ga, int m) {
    const int n = m / ga.L, r = m - n * ga.L, y = r / ga.Wo, x = r - y * ga.Wo;
    const int64_t base = static_cast<int64_t>(n) * ga.C * ga.H * ga.W;
    if (ga.mode == 0) return GatherRow{base, y * ga.s - ga.pt, x * ga.s - ga.pl};
    return GatherRow{base, y + ga.pt, x + ga.pl};
}

// Position of tap (kh, kw) of a gathered row, or false where it contributes 0.
// MODE: 0 patches, 1 either col2im gather, 2 col2im gather of stride 1, -1 read
// from ga.mode.
template <int MODE = -1>
__device__ __forceinline__ bool gather_tap(const Gather& ga, const GatherRow& gr, int kh, int kw,
                                           int* ih, int* iw) {
    if (MODE == 0 || (MODE < 0 && ga.mode == 0)) {
        *ih = gr.ih0 + kh;
        *iw = gr.iw0 + kw;
        return *ih >= 0 && *ih < ga.H && *iw >= 0 && *iw < ga.W;
    }
    const int ohn = gr.ih0 - kh, own = gr.iw0 - kw;
    if (MODE == 2 || ga.s == 1) {  // both gathers are the adjoint of the patches; no division
        *ih = ohn;
        *iw = own;
        return ohn >= 0 && ohn < ga.H && own >= 0 && own < ga.W;
    }
    const int oh = ohn / ga.s, ow = own / ga.s;  // C division truncates toward zero
    *ih = oh;
    *iw = ow;
    const bool okh = (ohn % ga.s == 0) && oh >= 0 && oh < ga.H && (ga.mode == 1 || ohn >= 0);
    const bool okw = ow >= 0 && ow < ga.W && (ga.mode == 1 || (own >= 0 && own % ga.s == 0));
    return okh && okw;
}

// Offset of reduction element r of a gathered row, or -1 where it contributes 0.
__device__ __forceinline__ int64_t gather_off(const Gather& ga, const GatherRow& gr, int r) {
    const int tap = r / ga.C, c = r - tap * ga.C, kh = tap / ga.k, kw = tap - kh * ga.k;
    int ih, iw;
    if (!gather_tap(ga, gr, kh, kw, &ih, &iw)) return -1;
    if (ga.nhwc) return gr.base + (static_cast<int64_t>(ih) * ga.W + iw) * ga.C + c;
    return gr.base + (static_cast<int64_t>(c) * ga.H + ih) * ga.W + iw;
}

struct GemmArgs {
    const float *x, *y;
    RowMap arow;
    int64_t ak;
    int ones_row;
    int64_t a_bs;
    Gather ga;
    const float *u, *v;
    RowMap brow;
    int64_t bn;
    int64_t b_bs;
    float *o0, *o1;
    RowMap orow;
    int64_t on;
    int64_t o_bs;
    const float *bias0, *bias1;
    float scale0, scale1;
    int M, N, Kr;
    int splits, kchunk;
    float* ws;
    ParamEpi pe;
    // Tensor-core path only: B operand tiles prepared by tc_pack_b for an N tile
    // of 2*bpk_nc columns (null = the kernel forms them from u, v); bpk_nkb
    // K-blocks of 8 reduction elements per column chunk.
    const char* bpk;
    int bpk_nc, bpk_nkb;
};

__device__ __forceinline__ void param_epilogue(int r, int c, float g0, float g1,
                                               const ParamEpi& p) {
    const int64_t rc = static_cast<int64_t>(r) * p.N + c;
    if (p.mode == TAGI_WGRAD_SUMS) {
        p.out_m[rc] = g0;
        p.out_S[rc] = g1;
        return;
    }
    const bool bias = (r == p.K);
    const int64_t w = bias ? c : rc;
    float* mp = bias ? p.mb : p.mw;
    float* Sp = bias ? p.Sb : p.Sw;
    const float S = Sp[w];
    const float dm = S * g0;
    const float dS = (S * S) * g1;
    if (p.mode == TAGI_WGRAD_DELTAS) {
        (bias ? p.out_mb : p.out_m)[w] = dm;
        (bias ? p.out_Sb : p.out_S)[w] = dS;
        return;
    }
    float m = mp[w], Sn = S;
    capped_pair(m, Sn, dm, dS, p.cap);
    mp[w] = m;
    Sp[w] = Sn;
}


// tcgen05 path (gemm_tc.cu). tc_pick returns the N tile (0 = use CUDA cores);
// with `fill` it narrows the tile when the grid would leave most SMs idle (for
// launches that do not fill the machine with split reductions).
int tc_pick(int vm, int M, int N, int Kr, int batch, bool fill = true);
int tc_launch(const GemmArgs& g, int vm, bool mean, int epi, int bn, int batch, cudaStream_t st,
              const char* what);
// Bytes of the prepared B tiles of a contraction with N output columns,
// reduction Kr and N tile bn (bn = 128 bounds the others), and the kernel that
// writes them into `dst` (256-byte aligned) and points g.bpk there.
size_t tc_pack_bytes(int vm, int N, int Kr, int bn);
int tc_pack_b(GemmArgs& g, int vm, int bn, void* dst, cudaStream_t st, const char* what);
constexpr int kTcBM = 128;

}  // namespace tagi
