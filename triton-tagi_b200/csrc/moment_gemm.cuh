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

struct GemmArgs {
    const float *x, *y;
    RowMap arow;
    int64_t ak;
    int ones_row;
    int64_t a_bs;
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
