// Gaussian embedding lookup and its parameter sums, and the positional-encoding
// add (triton_tagi/layers/embedding.py:88-151, positional_encoding.py:57-62).
//
// Token ids arrive as floats (the reference casts `ma.long()`, truncating toward
// zero). Ids outside [0, V) and the padding id give zero rows in the forward and
// contribute nothing to the sums (the reference's device indexing would abort the
// context on an out-of-range id; here no access is made).
//
// The sums are deterministic: one CTA per (vocabulary row, column slice) scans
// the token ids in order and adds the matching delta rows in token order, so a
// row's sum is the same sequence of fp32 additions as the reference's CPU
// index_add (product rounded, then added). The scan is O(V x tokens) id compares
// (cheap for the vocabularies of this path: 64 rows x 16384 tokens); the loads of
// the matching rows are issued ahead of the ordered adds.

#include <cstdint>

#include "common.cuh"
#include "tagi_b200.h"

namespace tagi {
namespace {

__device__ __forceinline__ int token_id(float x, int64_t V, int64_t pad) {
    // ids beyond int range are out of range anyway; keep the cast defined
    if (!(x > -1.0f && x < static_cast<float>(V))) return -1;
    const int c = static_cast<int>(x);  // truncation toward zero, as .long()
    return (c == pad) ? -1 : c;
}

// One thread per (token, 4 columns) when D % 4 == 0, else per (token, column).
template <bool V4>
__global__ void embedding_fwd_kernel(const float* idx, const float* mw, const float* Sw,
                                     float* mz, float* Sz, int64_t n, int64_t V, int64_t D,
                                     int64_t pad) {
    const int64_t per = V4 ? D / 4 : D;
    const int64_t total = n * per;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / per, j = i - t * per;
        const int v = token_id(idx[t], V, pad);
        if (V4) {
            float4 m = make_float4(0.f, 0.f, 0.f, 0.f), s = m;
            if (v >= 0) {
                m = __ldg(reinterpret_cast<const float4*>(mw + v * D) + j);
                s = __ldg(reinterpret_cast<const float4*>(Sw + v * D) + j);
            }
            reinterpret_cast<float4*>(mz + t * D)[j] = m;
            reinterpret_cast<float4*>(Sz + t * D)[j] = s;
        } else {
            mz[t * D + j] = v >= 0 ? mw[v * D + j] : 0.f;
            Sz[t * D + j] = v >= 0 ? Sw[v * D + j] : 0.f;
        }
    }
}

constexpr int kEmbIds = 1024;  // token ids staged per pass
constexpr int kEmbCols = 256;  // columns per CTA (one per thread)
constexpr int kEmbAhead = 8;   // delta rows loaded ahead of the ordered adds

// CTA (v, slice): columns slice*256 .. +255 of vocabulary row v. Sums mode
// (Sw == nullptr): out = sum dm, sum dS over the row's tokens; deltas mode:
// out_m = sum dm*Sw[v], out_S = sum (dS*Sw[v])*Sw[v] (the reference's product
// order; each product rounded, then added, in token order). Per pass of
// kEmbIds token ids, the positions of the row's tokens are compacted in token
// order (warp ballots, then the warps' counts in warp order); each thread then
// loads kEmbAhead delta rows at a time before adding them in that order.
__global__ void __launch_bounds__(kEmbCols) embedding_bwd_kernel(
    const float* idx, const float* dm, const float* dS, const float* Sw, int64_t n, int64_t V,
    int64_t D, int64_t pad, float* out_m, float* out_S) {
    __shared__ int pos[kEmbIds];
    __shared__ int wcount[kEmbCols / 32 + 1];
    const int v = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kWarps = kEmbCols / 32;
    const int64_t col = static_cast<int64_t>(blockIdx.y) * kEmbCols + threadIdx.x;
    const bool on = col < D;
    const float w = (Sw && on) ? Sw[v * D + col] : 1.f;
    float am = 0.f, aS = 0.f;
    for (int64_t t0 = 0; t0 < n; t0 += kEmbIds) {
        const int cnt = static_cast<int>(n - t0 < kEmbIds ? n - t0 : kEmbIds);
        // each warp owns kEmbIds / kWarps consecutive ids of the pass
        constexpr int kPer = kEmbIds / kWarps;
        const int base = warp * kPer;
        int mine = 0;
        for (int j = 0; j < kPer; j += 32) {
            const int i = base + j + lane;
            const bool hit = i < cnt && token_id(idx[t0 + i], V, pad) == v;
            mine += __popc(__ballot_sync(0xffffffffu, hit));
        }
        if (lane == 0) wcount[warp] = mine;
        __syncthreads();
        if (threadIdx.x == 0) {
            int run = 0;
            for (int k = 0; k < kWarps; ++k) {
                const int c = wcount[k];
                wcount[k] = run;
                run += c;
            }
            wcount[kWarps] = run;
        }
        __syncthreads();
        int at = wcount[warp];
        for (int j = 0; j < kPer; j += 32) {
            const int i = base + j + lane;
            const bool hit = i < cnt && token_id(idx[t0 + i], V, pad) == v;
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (hit) pos[at + __popc(m & ((1u << lane) - 1u))] = i;
            at += __popc(m);
        }
        __syncthreads();
        const int total = wcount[kWarps];
        if (on) {
            for (int k0 = 0; k0 < total; k0 += kEmbAhead) {
                float xm[kEmbAhead], xs[kEmbAhead];
#pragma unroll
                for (int u = 0; u < kEmbAhead; ++u) {
                    if (k0 + u < total) {
                        const int64_t o = (t0 + pos[k0 + u]) * D + col;
                        xm[u] = dm[o];
                        xs[u] = dS[o];
                    }
                }
#pragma unroll
                for (int u = 0; u < kEmbAhead; ++u) {
                    if (k0 + u < total) {
                        if (Sw) {
                            am = __fadd_rn(am, __fmul_rn(xm[u], w));
                            aS = __fadd_rn(aS, __fmul_rn(__fmul_rn(xs[u], w), w));
                        } else {
                            am = __fadd_rn(am, xm[u]);
                            aS = __fadd_rn(aS, xs[u]);
                        }
                    }
                }
            }
        }
        __syncthreads();  // pos and wcount are rewritten by the next pass
    }
    if (on) {
        out_m[v * D + col] = am;
        out_S[v * D + col] = aS;
    }
}

// out[r][d] = ma[r][d] + pe[r % S][d] over rows r of (B*S, D).
__global__ void positional_add_kernel(const float* ma, const float* pe, float* out, int64_t rows,
                                      int64_t S, int64_t D) {
    const int64_t total = rows * D;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / D, d = i - r * D;
        out[i] = ma[i] + pe[(r % S) * D + d];
    }
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" int tagi_embedding_forward(const float* idx, const float* mw, const float* Sw,
                                      float* mz, float* Sz, int64_t n, int64_t V, int64_t D,
                                      int64_t padding_idx, void* stream) {
    const char* what = "tagi_embedding_forward";
    TAGI_REQUIRE(n >= 0 && V >= 1 && D >= 1 && V <= INT32_MAX, TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (n == 0) return TAGI_OK;
    TAGI_REQUIRE(idx && mw && Sw && mz && Sz, TAGI_E_BAD_ARG, "%s: null pointer", what);
    const uintptr_t al = reinterpret_cast<uintptr_t>(mw) | reinterpret_cast<uintptr_t>(Sw) |
                         reinterpret_cast<uintptr_t>(mz) | reinterpret_cast<uintptr_t>(Sz);
    const bool v4 = D % 4 == 0 && (al & 15) == 0;
    const int64_t work = n * (v4 ? D / 4 : D);
    if (v4)
        embedding_fwd_kernel<true><<<grid_1d(work, 256), 256, 0, as_stream(stream)>>>(
            idx, mw, Sw, mz, Sz, n, V, D, padding_idx);
    else
        embedding_fwd_kernel<false><<<grid_1d(work, 256), 256, 0, as_stream(stream)>>>(
            idx, mw, Sw, mz, Sz, n, V, D, padding_idx);
    return check_launch(what);
}

extern "C" int tagi_embedding_backward(const float* idx, const float* dmz, const float* dSz,
                                       const float* Sw, int64_t n, int64_t V, int64_t D,
                                       int64_t padding_idx, int mode, float* out_m, float* out_S,
                                       void* stream) {
    const char* what = "tagi_embedding_backward";
    TAGI_REQUIRE(n >= 0 && V >= 1 && D >= 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    TAGI_REQUIRE(mode == TAGI_WGRAD_SUMS || mode == TAGI_WGRAD_DELTAS, TAGI_E_BAD_ARG,
                 "%s: mode must be TAGI_WGRAD_SUMS or TAGI_WGRAD_DELTAS", what);
    TAGI_REQUIRE(out_m && out_S && (n == 0 || (idx && dmz && dSz)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    TAGI_REQUIRE(mode == TAGI_WGRAD_SUMS || Sw, TAGI_E_BAD_ARG, "%s: deltas need Sw", what);
    const int64_t slices = (D + kEmbCols - 1) / kEmbCols;
    TAGI_REQUIRE(V <= INT32_MAX && slices <= 65535, TAGI_E_UNSUPPORTED, "%s: sizes beyond the grid",
                 what);
    const dim3 grid(static_cast<unsigned>(V), static_cast<unsigned>(slices), 1);
    embedding_bwd_kernel<<<grid, kEmbCols, 0, as_stream(stream)>>>(
        idx, dmz, dSz, mode == TAGI_WGRAD_DELTAS ? Sw : nullptr, n, V, D, padding_idx, out_m,
        out_S);
    return check_launch(what);
}

extern "C" int tagi_positional_add(const float* ma, const float* pe, float* out, int64_t rows,
                                   int64_t S, int64_t D, void* stream) {
    const char* what = "tagi_positional_add";
    TAGI_REQUIRE(rows >= 0 && S >= 1 && D >= 1, TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (rows == 0) return TAGI_OK;
    TAGI_REQUIRE(ma && pe && out, TAGI_E_BAD_ARG, "%s: null pointer", what);
    positional_add_kernel<<<grid_1d(rows * D, 256), 256, 0, as_stream(stream)>>>(ma, pe, out,
                                                                                 rows, S, D);
    return check_launch(what);
}
