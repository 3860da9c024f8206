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

// Implicit patches on the A side (convolutions without a patch matrix):
// A[m][r] = x[n][c][oh*s - pt + kh][ow*s - pl + kw], zero outside the input,
// for rows m = (n, oh, ow) over N x Ho x Wo and reduction index r = tap*C + c
// with tap = kh*k + kw. Taps outermost: 8 consecutive reduction elements then
// share one tap (for C a multiple of 8), i.e. one bounds test and 8 addresses
// a channel plane apart. The B operand is read in the same (tap, c) order.
struct Gather {
    int on;              // 1: A is gathered; arow and ak are unused
    int C, H, W;         // input channels and size (NCHW)
    int Wo, L;           // output width, output pixels per image
    int k, s, pt, pl;    // kernel size, stride, top and left padding
};

// One output pixel's image base and input origin.
struct GatherRow {
    int64_t base;
    int ih0, iw0;
};

__device__ __forceinline__ GatherRow gather_row(const Gather& ga, int m) {
    const int n = m / ga.L, r = m - n * ga.L, oh = r / ga.Wo, ow = r - oh * ga.Wo;
    return GatherRow{static_cast<int64_t>(n) * ga.C * ga.H * ga.W, oh * ga.s - ga.pt,
                     ow * ga.s - ga.pl};
}

// Offset of reduction element r of a gathered row, or -1 where the patch lies
// outside the input.
__device__ __forceinline__ int64_t gather_off(const Gather& ga, const GatherRow& gr, int r) {
    const int tap = r / ga.C, c = r - tap * ga.C, kh = tap / ga.k, kw = tap - kh * ga.k;
    const int ih = gr.ih0 + kh, iw = gr.iw0 + kw;
    if (ih < 0 || ih >= ga.H || iw < 0 || iw >= ga.W) return -1;
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


// tcgen05 path (gemm_tc.cu). tc_pick returns the N tile (0 = use CUDA cores).
int tc_pick(int vm, int M, int N, int Kr, int batch);
int tc_launch(const GemmArgs& g, int vm, bool mean, int epi, int bn, int batch, cudaStream_t st,
              const char* what);
constexpr int kTcBM = 128;

}  // namespace tagi
