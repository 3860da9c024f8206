// Moment contractions on CUDA cores (fp32 FMA, the reference's arithmetic).
//
// Every contraction on the TAGI path has two accumulators over one shared
// reduction: a mean product acc0 += x*u and a variance product acc1. Three
// variance forms cover all of them:
//   FULL : acc1 += x^2 v + y (u^2 + v)   Linear/Conv forward, bmm_tagi_var
//   RSQ  : acc1 += y u^2                 backward delta, bmm_shared_right
//   LSQ  : acc1 += x^2 v                 weight gradient, bmm_shared_left
// The A side (x, y) is an M x Kr view whose rows may be "row-split" (NCHW
// tensors read in place); the B side (u, v) is Kr x N whose reduction index
// may be row-split. Squares are formed once per element while staging tiles
// in shared memory. Large reductions with few output tiles (weight gradients
// of convolutions) are split over the reduction and finished by a fixed-order
// reduce kernel, so results are deterministic.
#include <algorithm>
#include <climits>
#include <mutex>

#include "common.cuh"
#include "moment_gemm.cuh"

namespace tagi {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256, PAD = 4;

template <int VM>
struct Needs {
    static constexpr bool y = (VM == FULL || VM == RSQ);
    static constexpr bool v = (VM == FULL || VM == LSQ);
    static constexpr int a_tiles = (VM == FULL) ? 3 : 2;
    static constexpr int b_tiles = (VM == FULL) ? 3 : 2;
};

template <int VM, bool MEAN, int EPI>
__global__ void __launch_bounds__(NT) moment_gemm_kernel(const GemmArgs g) {
    using Nd = Needs<VM>;
    __shared__ __align__(16) float As[Nd::a_tiles][BK][BM + PAD];
    __shared__ __align__(16) float Bs[Nd::b_tiles][BK][BN + PAD];

    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int batch = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
    const int kbeg = split * g.kchunk;
    const int kend = min(g.Kr, kbeg + g.kchunk);

    const float* x = g.x + batch * g.a_bs;
    const float* y = Nd::y ? g.y + batch * g.a_bs : nullptr;
    const float* u = g.u + batch * g.b_bs;
    const float* v = Nd::v ? g.v + batch * g.b_bs : nullptr;
    const bool a_kcontig = (g.ak == 1);
    const bool b_ncontig = (g.bn == 1);

    int a_mm[4], a_kk[4], b_nn[4], b_kk[4];
    int64_t a_off[4], b_col[4];
    bool a_ok[4], a_one[4], b_ok[4];
    GatherRow a_gr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int e = tid + i * NT;
        if (a_kcontig) { a_kk[i] = e % BK; a_mm[i] = e / BK; }
        else           { a_mm[i] = e % BM; a_kk[i] = e / BM; }
        const int row = m0 + a_mm[i];
        a_ok[i] = row < g.M;
        a_one[i] = (row == g.ones_row);
        a_off[i] = (a_ok[i] && !a_one[i] && !g.ga.on) ? g.arow.off(row) : 0;
        if (g.ga.on) a_gr[i] = gather_row(g.ga, a_ok[i] ? row : 0);
        if (b_ncontig) { b_nn[i] = e % BN; b_kk[i] = e / BN; }
        else           { b_kk[i] = e % BK; b_nn[i] = e / BK; }
        const int col = n0 + b_nn[i];
        b_ok[i] = col < g.N;
        b_col[i] = b_ok[i] ? static_cast<int64_t>(col) * g.bn : 0;
    }

    float rx[4], ry[4], ru[4], rv[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = k0 + a_kk[i];
            bool ok = a_ok[i] && k < kend;
            int64_t o;
            if (g.ga.on) {
                o = ok ? gather_off(g.ga, a_gr[i], k) : -1;
                ok = o >= 0;
            } else {
                o = a_off[i] + static_cast<int64_t>(k) * g.ak;
            }
            rx[i] = ok ? (a_one[i] ? 1.f : __ldg(x + o)) : 0.f;
            if (Nd::y) ry[i] = (ok && !a_one[i]) ? __ldg(y + o) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = k0 + b_kk[i];
            const bool ok = b_ok[i] && k < kend;
            const int64_t o = ok ? g.brow.off(k) + b_col[i] : 0;
            ru[i] = ok ? __ldg(u + o) : 0.f;
            if (Nd::v) rv[i] = ok ? __ldg(v + o) : 0.f;
        }
    };
    auto store = [&]() {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            As[0][a_kk[i]][a_mm[i]] = rx[i];
            if (VM == FULL) {
                As[1][a_kk[i]][a_mm[i]] = rx[i] * rx[i];
                As[2][a_kk[i]][a_mm[i]] = ry[i];
            } else if (VM == RSQ) {
                As[1][a_kk[i]][a_mm[i]] = ry[i];
            } else {
                As[1][a_kk[i]][a_mm[i]] = rx[i] * rx[i];
            }
            Bs[0][b_kk[i]][b_nn[i]] = ru[i];
            if (VM == FULL) {
                Bs[1][b_kk[i]][b_nn[i]] = rv[i];
                Bs[2][b_kk[i]][b_nn[i]] = ru[i] * ru[i] + rv[i];
            } else if (VM == RSQ) {
                Bs[1][b_kk[i]][b_nn[i]] = ru[i] * ru[i];
            } else {
                Bs[1][b_kk[i]][b_nn[i]] = rv[i];
            }
        }
    };

    float acc0[4][4], acc1[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc0[i][j] = acc1[i][j] = 0.f;

    if (kbeg < kend) load(kbeg);
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
        __syncthreads();
        store();
        __syncthreads();
        if (k0 + BK < kend) load(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[0][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[1][kk][ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[0][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[1][kk][tx * 4]);
            const float av0[4] = {a0.x, a0.y, a0.z, a0.w}, av1[4] = {a1.x, a1.y, a1.z, a1.w};
            const float bv0[4] = {b0.x, b0.y, b0.z, b0.w}, bv1[4] = {b1.x, b1.y, b1.z, b1.w};
            if (VM == FULL) {
                const float4 a2 = *reinterpret_cast<const float4*>(&As[2][kk][ty * 4]);
                const float4 b2 = *reinterpret_cast<const float4*>(&Bs[2][kk][tx * 4]);
                const float av2[4] = {a2.x, a2.y, a2.z, a2.w}, bv2[4] = {b2.x, b2.y, b2.z, b2.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (MEAN) acc0[i][j] = fmaf(av0[i], bv0[j], acc0[i][j]);
                        acc1[i][j] = fmaf(av1[i], bv1[j], acc1[i][j]);
                        acc1[i][j] = fmaf(av2[i], bv2[j], acc1[i][j]);
                    }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (MEAN) acc0[i][j] = fmaf(av0[i], bv0[j], acc0[i][j]);
                        acc1[i][j] = fmaf(av1[i], bv1[j], acc1[i][j]);
                    }
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = m0 + ty * 4 + i;
        if (r >= g.M) continue;
        const int64_t ro = (EPI == EPI_STORE) ? g.orow.off(r) + batch * g.o_bs : 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = n0 + tx * 4 + j;
            if (c >= g.N) continue;
            if (EPI == EPI_STORE) {
                const int64_t o = ro + static_cast<int64_t>(c) * g.on;
                if (MEAN && g.o0) g.o0[o] = g.scale0 * acc0[i][j] + (g.bias0 ? g.bias0[c] : 0.f);
                g.o1[o] = g.scale1 * acc1[i][j] + (g.bias1 ? g.bias1[c] : 0.f);
            } else if (EPI == EPI_PARTIAL) {
                const int64_t mn = static_cast<int64_t>(g.M) * g.N;
                const int64_t o = static_cast<int64_t>(r) * g.N + c;
                g.ws[(2 * split) * mn + o] = acc0[i][j];
                g.ws[(2 * split + 1) * mn + o] = acc1[i][j];
            } else {
                param_epilogue(r, c, acc0[i][j], acc1[i][j], g.pe);
            }
        }
    }
}

// Sums split-K partials in split order, then stores or applies the parameter epilogue.
// Output idx (row-major over M x N) of a split reduction whose totals are g0, g1:
// the parameter epilogue or the scaled, biased store.
__device__ __forceinline__ void finish_one(const GemmArgs& g, int param, int64_t idx, float g0,
                                           float g1) {
    const int r = static_cast<int>(idx / g.N), c = static_cast<int>(idx % g.N);
    if (param) {
        param_epilogue(r, c, g0, g1, g.pe);
    } else {
        const int64_t o = g.orow.off(r) + static_cast<int64_t>(c) * g.on;
        if (g.o0) g.o0[o] = g.scale0 * g0 + (g.bias0 ? g.bias0[c] : 0.f);
        g.o1[o] = g.scale1 * g1 + (g.bias1 ? g.bias1[c] : 0.f);
    }
}

// Partials of eight splits are loaded before they are added (in split order,
// so the sums are the same as one at a time): one load latency per eight
// splits instead of one per split.
// bsums (optional): the bias row `brow` from column sums computed elsewhere,
// as bias_given_kernel writes it.
__global__ void splitk_finish_kernel(const GemmArgs g, int param, const double* bsums, int brow) {
    constexpr int kAhead = 8;
    const int64_t mn = static_cast<int64_t>(g.M) * g.N;
    const float* ws = g.ws;
    if (bsums != nullptr)
        for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < g.N; n += gridDim.x * blockDim.x)
            finish_one(g, param, static_cast<int64_t>(brow) * g.N + n,
                       static_cast<float>(bsums[n]), static_cast<float>(bsums[g.N + n]));
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < mn;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float g0 = 0.f, g1 = 0.f;
        int s = 0;
        for (; s + kAhead <= g.splits; s += kAhead) {
            float a[kAhead], b[kAhead];
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                a[u] = __ldg(ws + (2 * static_cast<int64_t>(s + u)) * mn + idx);
                b[u] = __ldg(ws + (2 * static_cast<int64_t>(s + u) + 1) * mn + idx);
            }
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                g0 += a[u];
                g1 += b[u];
            }
        }
        for (; s < g.splits; ++s) {
            g0 += ws[(2 * static_cast<int64_t>(s)) * mn + idx];
            g1 += ws[(2 * static_cast<int64_t>(s) + 1) * mn + idx];
        }
        finish_one(g, param, idx, g0, g1);
    }
}

// The same for hundreds of splits over few outputs: 16 outputs per CTA, the
// splits dealt round-robin to 16 thread groups, then the 16 group totals added
// in group order (a fixed order: deterministic).
__global__ void __launch_bounds__(256) splitk_finish_wide_kernel(const GemmArgs g, int param) {
    __shared__ float red[2][16][17];
    const int64_t mn = static_cast<int64_t>(g.M) * g.N;
    const int o = threadIdx.x & 15, grp = threadIdx.x >> 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * 16 + o;
    float g0 = 0.f, g1 = 0.f;
    if (idx < mn) {
#pragma unroll 4
        for (int s = grp; s < g.splits; s += 16) {
            g0 += g.ws[(2 * static_cast<int64_t>(s)) * mn + idx];
            g1 += g.ws[(2 * static_cast<int64_t>(s) + 1) * mn + idx];
        }
    }
    red[0][grp][o] = g0;
    red[1][grp][o] = g1;
    __syncthreads();
    if (grp == 0 && idx < mn) {
        float t0 = 0.f, t1 = 0.f;
        for (int j = 0; j < 16; ++j) {
            t0 += red[0][j][o];
            t1 += red[1][j][o];
        }
        finish_one(g, param, idx, t0, t1);
    }
}

inline int cdiv(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Reduction split for output grids too small to fill the GPU, for the kernel
// (tensor-core or CUDA-core tiles) that will run the shape.
void choose_splits(int M, int N, int Kr, int batch, int* splits, int* kchunk, int* bn_tc) {
    const int tc = tc_pick(LSQ, M, N, Kr, batch, false);  // splits fill the machine
    int s = 1;
    if (tc) {
        // Tensor cores: CTAs come in pairs of 256 rows. Pick the split count that
        // minimises waves x (K-blocks per CTA + the cost of one partial epilogue,
        // about 8 K-blocks), i.e. fills the last wave without splitting needlessly.
        const int64_t ctas = 2 * static_cast<int64_t>(cdiv(M, 256)) * cdiv(N, tc) * batch;
        const int smax = std::min(64, std::max(1, Kr / (BK * 8)));
        if (batch == 1 && ctas < 2 * kNumSMs) {
            int64_t best = -1;
            for (int t = 1; t <= smax; ++t) {
                const int64_t waves = (ctas * t + kNumSMs - 1) / kNumSMs;
                const int64_t cost = waves * (cdiv(Kr, t * BK) + 8);
                if (best < 0 || cost < best) {
                    best = cost;
                    s = t;
                }
            }
        }
    } else {
        const int tiles = cdiv(M, BM) * cdiv(N, BN) * batch;
        if (batch == 1 && tiles < 2 * kNumSMs) {
            s = cdiv(2 * kNumSMs, tiles);
            s = std::min(s, std::max(1, Kr / (BK * 8)));
            s = std::min(s, 64);
        }
    }
    int chunk = cdiv(cdiv(Kr, s), BK) * BK;
    if (chunk < BK) chunk = BK;
    *splits = cdiv(Kr, chunk);
    if (*splits < 1) *splits = 1;
    *kchunk = chunk;
    *bn_tc = tc;
}

template <int VM, bool MEAN, int EPI>
int launch_simt(const GemmArgs& g, int batch, cudaStream_t st, const char* what) {
    if (g.M == 0 || g.N == 0) return TAGI_OK;
    dim3 grid(cdiv(g.N, BN), cdiv(g.M, BM), batch * g.splits);
    TAGI_REQUIRE(grid.y <= 65535 && grid.z <= 65535, TAGI_E_UNSUPPORTED, "%s: grid too large",
                 what);
    moment_gemm_kernel<VM, MEAN, EPI><<<grid, NT, 0, st>>>(g);
    return check_launch(what);
}

// Runs a contraction on the tensor cores when the shape is large enough
// (tc_pick), on CUDA cores otherwise. `bn_tc` forces the choice made by a
// planner that already sized a split-K workspace for it.
template <int VM, bool MEAN, int EPI>
int launch(const GemmArgs& g, int batch, cudaStream_t st, const char* what, int bn_tc = -1) {
    if (bn_tc < 0) bn_tc = tc_pick(VM, g.M, g.N, g.Kr, batch);
    if (bn_tc > 0) return tc_launch(g, VM, MEAN, EPI, bn_tc, batch, st, what);
    return launch_simt<VM, MEAN, EPI>(g, batch, st, what);
}

GemmArgs blank() {
    GemmArgs g{};
    g.ones_row = -1;
    g.scale0 = g.scale1 = 1.f;
    g.splits = 1;
    return g;
}

bool bad_size(int64_t v) { return v < 0 || v > (int64_t(1) << 31) - 1; }

// Prepared delta tiles pay when many output tiles along M (pairs of 256 weight
// rows) would each convert the same deltas: 8 or more.
size_t wgrad_pack_bytes(int Mo, int N, int Kr, int bn_tc) {
    if (bn_tc <= 0 || (Mo + 255) / 256 < 8) return 0;
    return tc_pack_bytes(LSQ, N, Kr, bn_tc);
}

// ---- weight sums of few weight rows over long reductions ---------------------
// A network's first convolution has few weight rows (C*k*k + 1: 28 for a 3x3
// RGB stem, 76 for 5x5) against a reduction over every output pixel. A
// tensor-core pair tile is 256 rows, so such a launch wastes 70-90 % of its
// MMAs and runs at a fraction of the rate of the other layers. Here one CTA
// owns a slice of the reduction and ALL Mo x N outputs in registers: thread
// (rg, cg) accumulates rows 4rg..4rg+3 x columns 4cg..4cg+3 of both sums in
// fp32 (sum a*u and sum a^2*v). Tiles of kSkTM reduction elements are staged
// transposed in shared memory ([k][row] and [k][column], padded pitches), so
// that each thread reads its 4 rows and 4 columns of one element as three
// 128-bit loads for 36 floating-point operations. Slices write split partials
// that splitk_finish_wide_kernel adds in a fixed order (deterministic) and
// passes to the store or parameter epilogue.
constexpr int kSkTM = 32;           // reduction elements per staged tile
constexpr int kSkMaxRows = 96;      // weight rows (incl. the bias row)
constexpr int kSkMaxCols = 64;      // output columns
constexpr int kSkAP = kSkMaxRows + 4;  // pitches = 4 mod 8 (staging stores)
constexpr int kSkBP = kSkMaxCols + 4;

bool skinny_ok(int Mo, int N, int Kr) {
    return Mo >= 1 && N >= 1 && Mo <= kSkMaxRows && N <= kSkMaxCols &&
           cdiv(Mo, 4) * cdiv(N, 4) <= 256 && Kr >= 16384;
}

void skinny_plan(int Kr, int* splits, int* chunk) {
    const int s = std::max(2, std::min(cdiv(Kr, 512), 4 * kNumSMs));
    *chunk = cdiv(cdiv(Kr, s), kSkTM) * kSkTM;
    *splits = cdiv(Kr, *chunk);
}

__global__ void __launch_bounds__(256) wgrad_skinny_kernel(const GemmArgs g) {
    __shared__ __align__(16) float sa[kSkTM][kSkAP];
    __shared__ __align__(16) float su[kSkTM][kSkBP];
    __shared__ __align__(16) float sv[kSkTM][kSkBP];
    constexpr int kNA = kSkMaxRows * kSkTM / 256;  // staged A elements per thread (max)
    constexpr int kNB = kSkMaxCols * kSkTM / 256;  // staged elements per delta operand
    const int Mo = g.M, N = g.N;
    const int RG = (Mo + 3) >> 2, CG = (N + 3) >> 2;
    const int tid = threadIdx.x;
    const bool active = tid < RG * CG;
    const int rg = active ? tid / CG : 0, cg = active ? tid - rg * CG : 0;
    const int kb = blockIdx.x * g.kchunk, ke = min(g.Kr, kb + g.kchunk);
    float am[4][4] = {}, aS[4][4] = {};
    // tile k0 .. k0+kSkTM-1 into registers: A rows up to 4*RG (zeros past Mo,
    // ones on the bias row), delta columns up to 4*CG (zeros past N)
    float ra[kNA], ru[kNB], rv[kNB];
    // staged element i = tid + 256 q is (row or column i / 32, element i % 32):
    // every element a thread stages lies at reduction index k0 + (tid % 32), rows
    // (columns) tid / 32 + 8 q
    const int ki_t = tid & (kSkTM - 1), rc0 = tid / kSkTM;
    static_assert(256 % kSkTM == 0, "staging layout");
    auto fetch = [&](int k0) {
        const int k = k0 + ki_t;
        const bool kin = k < ke;
        const int64_t ak = static_cast<int64_t>(k) * g.ak;
#pragma unroll
        for (int q = 0; q < kNA; ++q) {
            const int r = rc0 + q * (256 / kSkTM);
            float x = 0.f;
            if (kin && r < Mo)
                x = r == g.ones_row ? 1.f : __ldg(g.x + g.arow.off(r) + ak);
            ra[q] = x;
        }
        const int64_t bo = kin ? g.brow.off(k) : 0;
#pragma unroll
        for (int q = 0; q < kNB; ++q) {
            const int c = rc0 + q * (256 / kSkTM);
            float u = 0.f, v = 0.f;
            if (kin && c < N) {
                const int64_t o = static_cast<int64_t>(c) * g.bn + bo;
                u = __ldg(g.u + o);
                v = __ldg(g.v + o);
            }
            ru[q] = u;
            rv[q] = v;
        }
    };
    auto put = [&]() {
#pragma unroll
        for (int q = 0; q < kNA; ++q) {
            const int r = rc0 + q * (256 / kSkTM);
            if (r < 4 * RG) sa[ki_t][r] = ra[q];
        }
#pragma unroll
        for (int q = 0; q < kNB; ++q) {
            const int c = rc0 + q * (256 / kSkTM);
            if (c < 4 * CG) {
                su[ki_t][c] = ru[q];
                sv[ki_t][c] = rv[q];
            }
        }
    };
    // double buffering through registers: the next tile's loads are in flight
    // while this tile is summed
    if (kb < ke) fetch(kb);
    for (int k0 = kb; k0 < ke; k0 += kSkTM) {
        __syncthreads();  // the previous tile has been read
        put();
        __syncthreads();
        if (k0 + kSkTM < ke) fetch(k0 + kSkTM);
        if (active) {
            // elements past the slice end are staged as zeros and add nothing
#pragma unroll 8
            for (int ki = 0; ki < kSkTM; ++ki) {
                const float4 a = *reinterpret_cast<const float4*>(&sa[ki][4 * rg]);
                const float4 u = *reinterpret_cast<const float4*>(&su[ki][4 * cg]);
                const float4 v = *reinterpret_cast<const float4*>(&sv[ki][4 * cg]);
                const float ar[4] = {a.x, a.y, a.z, a.w}, ur[4] = {u.x, u.y, u.z, u.w};
                const float vr[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float a2 = ar[i] * ar[i];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        am[i][j] = fmaf(ar[i], ur[j], am[i][j]);
                        aS[i][j] = fmaf(a2, vr[j], aS[i][j]);
                    }
                }
            }
        }
    }
    if (!active) return;
    const int64_t mn = static_cast<int64_t>(Mo) * N;
    float* pm = g.ws + (2 * static_cast<int64_t>(blockIdx.x)) * mn;
    float* pS = pm + mn;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * rg + i;
        if (r >= Mo) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = 4 * cg + j;
            if (c < N) {
                pm[static_cast<int64_t>(r) * N + c] = am[i][j];
                pS[static_cast<int64_t>(r) * N + c] = aS[i][j];
            }
        }
    }
}

// Split plan of the weight sums: the skinny kernel above, or tensor-core / CUDA-
// core tiles (choose_splits). bn_tc = 0 for the skinny kernel.
void plan_wgrad(int Mo, int N, int Kr, int* splits, int* chunk, int* bn_tc, bool* skinny) {
    *skinny = skinny_ok(Mo, N, Kr);
    if (*skinny) {
        skinny_plan(Kr, splits, chunk);
        *bn_tc = 0;
        return;
    }
    choose_splits(Mo, N, Kr, 1, splits, chunk, bn_tc);
}

// ---- bias sums apart from the weight rows -----------------------------------
// The weight sums carry a bias as a row of ones after the K weight rows. When K
// is a multiple of 256 that row alone would open another 256-row tensor-core
// pair tile (513 rows: three tiles for the work of two), so the bias sums are
// then formed by a column-sum pass and the contraction runs on the K weight rows.
size_t wgrad_ws_total(int Mo, int N, int Kr);

bool bias_apart(int Mo, int N, int Kr, bool bias_row) {
    if (!bias_row || Mo < 2 || Kr < 1 || (Mo - 1) % 256 != 0) return false;
    int splits, chunk, bn_tc;
    bool skinny;
    plan_wgrad(Mo - 1, N, Kr, &splits, &chunk, &bn_tc, &skinny);
    return bn_tc > 0 && !skinny;
}

// Reduction slices of the column sums: enough CTAs of 32 columns to fill the
// machine twice, slices of at least 256 rows.
void bias_plan(int N, int Kr, int* slices, int* chunk) {
    int s = std::max(1, std::min(64, cdiv(2 * kNumSMs, cdiv(N, 32))));
    s = std::min(s, std::max(1, cdiv(Kr, 256)));
    *chunk = cdiv(Kr, s);
    *slices = cdiv(Kr, *chunk);
}

// Workspace of a weight-sum call with the bias apart: the weight rows' own
// workspace, then (256-byte aligned) the column-sum slices.
size_t bias_apart_bytes(int Mo, int N, int Kr, size_t* off) {
    int slices, chunk;
    bias_plan(N, Kr, &slices, &chunk);
    *off = (wgrad_ws_total(Mo - 1, N, Kr) + 255) / 256 * 256;
    return *off + sizeof(float) * 2ull * slices * static_cast<size_t>(N);
}

// CTA (32 columns, one reduction slice): thread (column c, row group r) adds
// rows r, r+8, ... of the slice, eight rows' loads in flight before their adds
// (the same order of additions); the 8 group totals are added in group order.
__global__ void __launch_bounds__(256) bias_sums_kernel(const GemmArgs g, int chunk, float* part) {
    constexpr int kAhead = 8;
    __shared__ float red[2][8][33];
    const int c = threadIdx.x & 31, r = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + c;
    const int m0 = blockIdx.y * chunk, m1 = min(g.Kr, m0 + chunk);
    float a = 0.f, b = 0.f;
    if (n < g.N) {
        const int64_t col = static_cast<int64_t>(n) * g.bn;
        int m = m0 + r;
        for (; m + 8 * (kAhead - 1) < m1; m += 8 * kAhead) {
            float xa[kAhead], xb[kAhead];
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                const int64_t o = col + g.brow.off(m + 8 * u);
                xa[u] = __ldg(g.u + o);
                xb[u] = __ldg(g.v + o);
            }
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                a += xa[u];
                b += xb[u];
            }
        }
        for (; m < m1; m += 8) {
            const int64_t o = col + g.brow.off(m);
            a += __ldg(g.u + o);
            b += __ldg(g.v + o);
        }
    }
    red[0][r][c] = a;
    red[1][r][c] = b;
    __syncthreads();
    if (r == 0 && n < g.N) {
        float ta = 0.f, tb = 0.f;
        for (int j = 0; j < 8; ++j) {
            ta += red[0][j][c];
            tb += red[1][j][c];
        }
        part[(2 * static_cast<int64_t>(blockIdx.y)) * g.N + n] = ta;
        part[(2 * static_cast<int64_t>(blockIdx.y) + 1) * g.N + n] = tb;
    }
}

// Adds the slices in order and applies the epilogue to output row `row`.
__global__ void bias_finish_kernel(const GemmArgs g, int slices, const float* part, int param,
                                   int row) {
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < g.N; n += gridDim.x * blockDim.x) {
        float ta = 0.f, tb = 0.f;
        for (int s = 0; s < slices; ++s) {
            ta += part[(2 * static_cast<int64_t>(s)) * g.N + n];
            tb += part[(2 * static_cast<int64_t>(s) + 1) * g.N + n];
        }
        finish_one(g, param, static_cast<int64_t>(row) * g.N + n, ta, tb);
    }
}

// The bias row from column sums computed elsewhere (float64 sums of the
// deltas: sums[n] of the means, sums[N + n] of the variances).
__global__ void bias_given_kernel(const GemmArgs g, const double* sums, int param, int row) {
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < g.N; n += gridDim.x * blockDim.x)
        finish_one(g, param, static_cast<int64_t>(row) * g.N + n, static_cast<float>(sums[n]),
                   static_cast<float>(sums[g.N + n]));
}

// Shared driver for the weight-gradient family (stores or parameter epilogue).
// The workspace must hold the split-reduction partials when a split is planned;
// room past them (256-byte aligned) takes the prepared B tiles (the deltas) of
// the tensor-core kernel.
// `bsums` (the bias row is the last of Mo): the bias row's sums are given.
// `brow_sums` (internal): the sums of the bias row Mo, which follows these Mo
// rows; the split finish writes it, else bias_given_kernel.
int run_wgrad(GemmArgs& g, int Mo, void* ws, size_t ws_bytes, bool param, cudaStream_t st,
              const char* what, const double* bsums = nullptr,
              const double* brow_sums = nullptr) {
    if (bsums != nullptr) {
        GemmArgs gw = g;
        gw.ones_row = -1;
        int rc = TAGI_OK;
        if (Mo > 1) {
            rc = run_wgrad(gw, Mo - 1, ws, ws_bytes, param, st, what, nullptr, bsums);
        } else {
            bias_given_kernel<<<grid_1d(g.N, 256), 256, 0, st>>>(g, bsums, param ? 1 : 0, Mo - 1);
            rc = check_launch(what);
        }
        g.M = Mo;
        return rc;
    }
    auto bias_row = [&]() -> int {  // the given bias row, where no finish pass writes it
        if (brow_sums == nullptr) return TAGI_OK;
        bias_given_kernel<<<grid_1d(g.N, 256), 256, 0, st>>>(g, brow_sums, param ? 1 : 0, Mo);
        return check_launch(what);
    };
    if (bias_apart(Mo, g.N, g.Kr, g.ones_row == Mo - 1)) {
        size_t off = 0;
        const size_t total = bias_apart_bytes(Mo, g.N, g.Kr, &off);
        if (ws != nullptr && ws_bytes >= total) {  // else: the ones row, as below
            int slices, chunk;
            bias_plan(g.N, g.Kr, &slices, &chunk);
            float* part = reinterpret_cast<float*>(static_cast<char*>(ws) + off);
            const unsigned cols = static_cast<unsigned>(cdiv(g.N, 32));
            bias_sums_kernel<<<dim3(cols, static_cast<unsigned>(slices)), 256, 0, st>>>(g, chunk,
                                                                                       part);
            int rc = check_launch(what);
            if (rc) return rc;
            bias_finish_kernel<<<grid_1d(g.N, 256), 256, 0, st>>>(g, slices, part, param ? 1 : 0,
                                                                  Mo - 1);
            rc = check_launch(what);
            if (rc) return rc;
            GemmArgs gw = g;
            gw.ones_row = -1;
            rc = run_wgrad(gw, Mo - 1, ws, off, param, st, what);
            g.M = Mo;
            return rc;
        }
    }
    int splits, chunk, bn_tc;
    bool skinny;
    plan_wgrad(Mo, g.N, g.Kr, &splits, &chunk, &bn_tc, &skinny);
    g.M = Mo;
    if (skinny) {
        const size_t part = sizeof(float) * 2ull * splits * static_cast<size_t>(Mo) * g.N;
        TAGI_REQUIRE(ws != nullptr && ws_bytes >= part, TAGI_E_WORKSPACE,
                     "%s: workspace of %zu bytes required, %zu given", what, part, ws_bytes);
        g.splits = splits;
        g.kchunk = chunk;
        g.ws = static_cast<float*>(ws);
        wgrad_skinny_kernel<<<splits, 256, 0, st>>>(g);
        int rc = check_launch(what);
        if (rc) return rc;
        const int64_t mn = static_cast<int64_t>(Mo) * g.N;  // <= 96 x 64
        splitk_finish_wide_kernel<<<static_cast<unsigned>((mn + 15) / 16), 256, 0, st>>>(
            g, param ? 1 : 0);
        rc = check_launch(what);
        return rc ? rc : bias_row();
    }
    const size_t need = splits > 1 ? sizeof(float) * 2ull * splits * static_cast<size_t>(Mo) * g.N : 0;
    const size_t pack_off = (need + 255) / 256 * 256;
    const size_t pack = wgrad_pack_bytes(Mo, g.N, g.Kr, bn_tc);
    if (pack > 0 && ws != nullptr && ws_bytes >= pack_off + pack) {
        const int rc = tc_pack_b(g, LSQ, bn_tc, static_cast<char*>(ws) + pack_off, st, what);
        if (rc) return rc;
    }
    if (splits > 1) {
        TAGI_REQUIRE(ws != nullptr && ws_bytes >= need, TAGI_E_WORKSPACE,
                     "%s: workspace of %zu bytes required, %zu given", what, need, ws_bytes);
        g.splits = splits;
        g.kchunk = chunk;
        g.ws = static_cast<float*>(ws);
        int rc = launch<LSQ, true, EPI_PARTIAL>(g, 1, st, what, bn_tc);
        if (rc) return rc;
        splitk_finish_kernel<<<grid_1d(static_cast<int64_t>(Mo) * g.N, 256), 256, 0, st>>>(
            g, param ? 1 : 0, brow_sums, Mo);
        return check_launch(what);
    }
    g.splits = 1;
    g.kchunk = g.Kr > 0 ? g.Kr : BK;
    const int rc = param ? launch<LSQ, true, EPI_PARAM>(g, 1, st, what, bn_tc)
                         : launch<LSQ, true, EPI_STORE>(g, 1, st, what, bn_tc);
    return rc ? rc : bias_row();
}

// Workspace of a store-epilogue contraction: split-reduction partials (when the
// output grid leaves SMs idle), then the prepared B tiles of the tensor-core
// kernel (sized for FULL, the larger of FULL and RSQ).
struct StorePlan {
    int splits, chunk, bn_split, bn_whole;
    size_t partials, pack;
};

StorePlan store_plan(int M, int N, int Kr) {
    StorePlan p{};
    choose_splits(M, N, Kr, 1, &p.splits, &p.chunk, &p.bn_split);
    p.bn_whole = tc_pick(FULL, M, N, Kr, 1);
    p.partials = p.splits > 1 ? (sizeof(float) * 2ull * p.splits * static_cast<size_t>(M) * N + 255) /
                                    256 * 256
                              : 0;
    p.pack = (p.bn_split > 0 || p.bn_whole > 0) ? tc_pack_bytes(FULL, N, Kr, 128) : 0;
    return p;
}

size_t store_ws_bytes(int M, int N, int Kr) {
    const StorePlan p = store_plan(M, N, Kr);
    return p.partials + p.pack;
}

// Store-epilogue contractions (forward, input deltas). With a caller workspace
// they split the reduction when the output grid leaves SMs idle and give the
// tensor-core kernel prepared B tiles; a smaller workspace (or none) drops the
// prepared tiles first, then the split (the workspace only buys speed).
template <int VM>
int run_store(GemmArgs& g, void* ws, size_t ws_bytes, cudaStream_t st, const char* what) {
    const StorePlan p = store_plan(g.M, g.N, g.Kr);
    char* w = static_cast<char*>(ws);
    if (w == nullptr) ws_bytes = 0;
    const bool split = p.splits > 1 && ws_bytes >= p.partials;
    const int bn = split ? p.bn_split : tc_pick(VM, g.M, g.N, g.Kr, 1);
    // Prepared B tiles pay for the forward, whose weight-side producers bound the
    // tensor-core kernel; the input-delta contraction forms its B side (the
    // weights, read row by row) faster than a separate pass prepares it.
    const size_t pack = (VM == FULL && bn > 0) ? tc_pack_bytes(VM, g.N, g.Kr, bn) : 0;
    const size_t pack_off = split ? p.partials : 0;
    if (pack > 0 && ws_bytes >= pack_off + pack) {
        const int rc = tc_pack_b(g, VM, bn, w + pack_off, st, what);
        if (rc) return rc;
    }
    if (split) {
        g.splits = p.splits;
        g.kchunk = p.chunk;
        g.ws = reinterpret_cast<float*>(w);
        int rc = launch<VM, true, EPI_PARTIAL>(g, 1, st, what, p.bn_split);
        if (rc) return rc;
        splitk_finish_kernel<<<grid_1d(static_cast<int64_t>(g.M) * g.N, 256), 256, 0, st>>>(
            g, 0, nullptr, 0);
        return check_launch(what);
    }
    g.splits = 1;
    g.kchunk = g.Kr > 0 ? g.Kr : BK;
    return launch<VM, true, EPI_STORE>(g, 1, st, what, bn);
}

// Split-reduction partials a weight-gradient call requires.
size_t wgrad_ws_bytes(int Mo, int N, int Kr) {
    int splits, chunk, bn_tc;
    bool skinny;
    plan_wgrad(Mo, N, Kr, &splits, &chunk, &bn_tc, &skinny);
    return (splits > 1 || skinny) ? sizeof(float) * 2ull * splits * static_cast<size_t>(Mo) * N : 0;
}

// The partials plus the optional prepared B tiles (what the size queries report).
size_t wgrad_ws_total(int Mo, int N, int Kr) {
    int splits, chunk, bn_tc;
    bool skinny;
    plan_wgrad(Mo, N, Kr, &splits, &chunk, &bn_tc, &skinny);
    const size_t need = wgrad_ws_bytes(Mo, N, Kr);
    const size_t pack = wgrad_pack_bytes(Mo, N, Kr, bn_tc);
    return pack > 0 ? (need + 255) / 256 * 256 + pack : need;
}

// Element i of the (K + bias) x N sums: param_epilogue needs its row only to
// tell the bias row (r == K) and to form r * N + c = i, so (when K N fits an
// int) the weight rows go as (0, i) and the bias row as (K, i - K N): no
// division per element.
__global__ void apply_sums_kernel(const float* gm, const float* gS, ParamEpi p, int64_t total) {
    const int64_t kn = static_cast<int64_t>(p.K) * p.N;
    const bool flat = kn + p.N <= INT_MAX;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool bias = i >= kn;
        if (flat)
            param_epilogue(bias ? p.K : 0, static_cast<int>(bias ? i - kn : i), gm[i], gS[i], p);
        else
            param_epilogue(static_cast<int>(i / p.N), static_cast<int>(i % p.N), gm[i], gS[i], p);
    }
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" int tagi_fused_var_forward(const float* ma, const float* Sa, const float* mw,
                                      const float* Sw, const float* Sb, float* Sz, int64_t M,
                                      int64_t N, int64_t K, int64_t stride_am, int64_t stride_ak,
                                      int64_t stride_wk, int64_t stride_wn, int64_t stride_cm,
                                      int64_t stride_cn, void* stream) {
    const char* what = "tagi_fused_var_forward";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(Sz && (K == 0 || (ma && Sa && mw && Sw)), TAGI_E_BAD_ARG, "%s: null pointer",
                 what);
    GemmArgs g = blank();
    g.x = ma; g.y = Sa; g.arow = plain_rows(stride_am); g.ak = stride_ak;
    g.u = mw; g.v = Sw; g.brow = plain_rows(stride_wk); g.bn = stride_wn;
    g.o1 = Sz; g.orow = plain_rows(stride_cm); g.on = stride_cn; g.bias1 = Sb;
    g.M = (int)M; g.N = (int)N; g.Kr = (int)K; g.kchunk = K > 0 ? (int)K : BK;
    return launch<FULL, false, EPI_STORE>(g, 1, as_stream(stream), what);
}

extern "C" int tagi_moment_forward(const float* ma, const float* Sa, int64_t a_div,
                                   int64_t a_outer, int64_t a_stride, int64_t a_kstride,
                                   const float* mw, const float* Sw, int64_t ldw, const float* mb,
                                   const float* Sb, float* mz, float* Sz, int64_t c_div,
                                   int64_t c_outer, int64_t c_stride, int64_t c_nstride, int64_t M,
                                   int64_t N, int64_t K, void* stream) {
    const char* what = "tagi_moment_forward";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && (K == 0 || (ma && Sa && mw && Sw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = ma; g.y = Sa; g.arow = RowMap{a_div, a_outer, a_stride}; g.ak = a_kstride;
    g.u = mw; g.v = Sw; g.brow = plain_rows(ldw); g.bn = 1;
    g.o0 = mz; g.o1 = Sz; g.orow = RowMap{c_div, c_outer, c_stride}; g.on = c_nstride;
    g.bias0 = mb; g.bias1 = Sb;
    g.M = (int)M; g.N = (int)N; g.Kr = (int)K; g.kchunk = K > 0 ? (int)K : BK;
    return launch<FULL, true, EPI_STORE>(g, 1, as_stream(stream), what);
}

extern "C" int tagi_backward_delta_view(const float* dmz, const float* dSz, int64_t d_div,
                                        int64_t d_outer, int64_t d_stride, int64_t d_nstride,
                                        const float* mw, int64_t ldw, float* d_ma, float* d_Sa,
                                        int64_t c_div, int64_t c_outer, int64_t c_stride,
                                        int64_t c_kstride, int64_t M, int64_t K, int64_t N,
                                        void* stream) {
    const char* what = "tagi_backward_delta_view";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || K == 0) return TAGI_OK;
    TAGI_REQUIRE(d_ma && d_Sa && (N == 0 || (dmz && dSz && mw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = dmz; g.y = dSz; g.arow = RowMap{d_div, d_outer, d_stride}; g.ak = d_nstride;
    // u[r = n, j = k] = mw[k, n]
    g.u = mw; g.brow = plain_rows(1); g.bn = ldw;
    g.o0 = d_ma; g.o1 = d_Sa; g.orow = RowMap{c_div, c_outer, c_stride}; g.on = c_kstride;
    g.M = (int)M; g.N = (int)K; g.Kr = (int)N; g.kchunk = N > 0 ? (int)N : BK;
    return launch<RSQ, true, EPI_STORE>(g, 1, as_stream(stream), what);
}

// Output size and top/left padding of a Conv2D (padding type 1: symmetric;
// 2: p on the right/bottom only), as triton_tagi/layers/conv2d.py computes them.
static void conv_geometry(int64_t H, int64_t W, int64_t k, int64_t s, int64_t p, int64_t pt,
                   int64_t* Ho, int64_t* Wo, int* top) {
    if (pt == 2 && p > 0) {
        *Ho = (H + p - k) / s + 1;
        *Wo = (W + p - k) / s + 1;
        *top = 0;
    } else {
        *Ho = (H + 2 * p - k) / s + 1;
        *Wo = (W + 2 * p - k) / s + 1;
        *top = static_cast<int>(p);
    }
}

extern "C" int tagi_conv2d_forward(const float* ma, const float* Sa, const float* mw,
                                   const float* Sw, const float* mb, const float* Sb, float* mz,
                                   float* Sz, int64_t N, int64_t C, int64_t H, int64_t W,
                                   int64_t Co, int64_t k, int64_t stride, int64_t padding,
                                   int64_t padding_type, int nhwc, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    const char* what = "tagi_conv2d_forward";
    TAGI_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && Co >= 0 && k >= 1 && stride >= 1 &&
                     padding >= 0 && (padding_type == 1 || padding_type == 2),
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    int64_t Ho, Wo;
    int top;
    conv_geometry(H, W, k, stride, padding, padding_type, &Ho, &Wo, &top);
    TAGI_REQUIRE(Ho >= 1 && Wo >= 1, TAGI_E_BAD_ARG, "%s: kernel larger than the padded input",
                 what);
    const int64_t L = Ho * Wo, M = N * L, Kr = C * k * k;
    TAGI_REQUIRE(!bad_size(M) && !bad_size(Co) && !bad_size(Kr) && !bad_size(N * C * H * W) &&
                     !bad_size(Co * L),
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (M == 0 || Co == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && mb && Sb && (Kr == 0 || (ma && Sa && mw && Sw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = ma; g.y = Sa;
    g.ga = Gather{1, 0, (int)C, (int)H, (int)W, (int)Wo, (int)L, (int)k, (int)stride, top, top,
                  nhwc ? 1 : 0};
    // B[co][tap*C + c] = mw[c*kk + tap][co]: the weight rows in (tap, c) order
    g.u = mw; g.v = Sw; g.brow = RowMap{C, Co, k * k * Co}; g.bn = 1;
    g.bias0 = mb; g.bias1 = Sb;
    // outputs straight into NCHW: row (n, l) -> n*Co*L + l, column c -> c*L
    g.o0 = mz; g.o1 = Sz; g.orow = RowMap{L, Co * L, 1}; g.on = L;
    g.M = (int)M; g.N = (int)Co; g.Kr = (int)Kr;
    return run_store<FULL>(g, workspace, workspace_bytes, as_stream(stream), what);
}

extern "C" int tagi_conv2d_backward_delta(const float* dmz, const float* dSz, const float* mw,
                                          float* d_ma, float* d_Sa, int64_t N, int64_t C,
                                          int64_t H, int64_t W, int64_t Co, int64_t k,
                                          int64_t stride, int64_t padding, int64_t padding_type,
                                          int col2im_mode, int nhwc, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    const char* what = "tagi_conv2d_backward_delta";
    TAGI_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && Co >= 0 && k >= 1 && stride >= 1 &&
                     padding >= 0 && (padding_type == 1 || padding_type == 2) &&
                     (col2im_mode == 0 || col2im_mode == 1),
                 TAGI_E_BAD_ARG, "%s: bad arguments", what);
    int64_t Ho, Wo;
    int top;
    conv_geometry(H, W, k, stride, padding, padding_type, &Ho, &Wo, &top);
    TAGI_REQUIRE(Ho >= 1 && Wo >= 1, TAGI_E_BAD_ARG, "%s: kernel larger than the padded input",
                 what);
    const int64_t HW = H * W, kk = k * k, M = N * HW, Kr = Co * kk;
    TAGI_REQUIRE(!bad_size(M) && !bad_size(C) && !bad_size(Kr) && !bad_size(C * HW) &&
                     !bad_size(N * Co * Ho * Wo) && !bad_size(C * kk * Co),
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (M == 0 || C == 0) return TAGI_OK;
    TAGI_REQUIRE(d_ma && d_Sa && (Kr == 0 || (dmz && dSz && mw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    // A: the col2im gather of the deltas (Co x Ho x Wo per image) for rows (n, h, w)
    // of the input, reduction (tap, co)
    g.x = dmz; g.y = dSz;
    g.ga = Gather{1, col2im_mode == 0 ? 1 : 2, (int)Co, (int)Ho, (int)Wo, (int)W, (int)HW,
                  (int)k, (int)stride, top, top, nhwc ? 1 : 0};
    // B[c][tap*Co + co] = mw[c*kk + tap][co]: the weight matrix read in place, row c
    // contiguous along the reduction
    g.u = mw; g.brow = plain_rows(1); g.bn = Kr;
    // outputs straight into NCHW: row (n, hw) -> n*C*HW + hw, column c -> c*HW
    g.o0 = d_ma; g.o1 = d_Sa; g.orow = RowMap{HW, C * HW, 1}; g.on = HW;
    g.M = (int)M; g.N = (int)C; g.Kr = (int)Kr;
    return run_store<RSQ>(g, workspace, workspace_bytes, as_stream(stream), what);
}

extern "C" size_t tagi_store_workspace_size(int64_t M, int64_t N, int64_t K) {
    if (bad_size(M) || bad_size(N) || bad_size(K)) return 0;
    return store_ws_bytes((int)M, (int)N, (int)K);
}

extern "C" int tagi_linear_forward(const float* ma, const float* Sa, const float* mw,
                                   const float* Sw, const float* mb, const float* Sb, float* mz,
                                   float* Sz, int64_t M, int64_t K, int64_t N, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    const char* what = "tagi_linear_forward";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(mz && Sz && (K == 0 || (ma && Sa && mw && Sw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = ma; g.y = Sa; g.arow = plain_rows(K); g.ak = 1;
    g.u = mw; g.v = Sw; g.brow = plain_rows(N); g.bn = 1;
    g.bias0 = mb; g.bias1 = Sb;
    g.o0 = mz; g.o1 = Sz; g.orow = plain_rows(N); g.on = 1;
    g.M = (int)M; g.N = (int)N; g.Kr = (int)K;
    return run_store<FULL>(g, workspace, workspace_bytes, as_stream(stream), what);
}

extern "C" int tagi_linear_backward_delta(const float* dmz, const float* dSz, const float* mw,
                                          float* d_ma, float* d_Sa, int64_t M, int64_t K,
                                          int64_t N, void* workspace, size_t workspace_bytes,
                                          void* stream) {
    const char* what = "tagi_linear_backward_delta";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || K == 0) return TAGI_OK;
    TAGI_REQUIRE(d_ma && d_Sa && (N == 0 || (dmz && dSz && mw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = dmz; g.y = dSz; g.arow = plain_rows(N); g.ak = 1;
    g.u = mw; g.brow = plain_rows(1); g.bn = N;  // u[r = k][j = n] = mw[k, n]
    g.o0 = d_ma; g.o1 = d_Sa; g.orow = plain_rows(K); g.on = 1;
    g.M = (int)M; g.N = (int)K; g.Kr = (int)N;
    return run_store<RSQ>(g, workspace, workspace_bytes, as_stream(stream), what);
}

extern "C" int tagi_fused_backward_delta(const float* dmz, const float* dSz, const float* mw,
                                         float* d_ma, float* d_Sa, int64_t M, int64_t K,
                                         int64_t N, int64_t stride_dm, int64_t stride_dn,
                                         int64_t stride_wk, int64_t stride_wn, int64_t stride_cm,
                                         int64_t stride_ck, void* stream) {
    const char* what = "tagi_fused_backward_delta";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (M == 0 || K == 0) return TAGI_OK;
    TAGI_REQUIRE(d_ma && d_Sa && (N == 0 || (dmz && dSz && mw)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = dmz; g.y = dSz; g.arow = plain_rows(stride_dm); g.ak = stride_dn;
    g.u = mw; g.brow = plain_rows(stride_wn); g.bn = stride_wk;
    g.o0 = d_ma; g.o1 = d_Sa; g.orow = plain_rows(stride_cm); g.on = stride_ck;
    g.M = (int)M; g.N = (int)K; g.Kr = (int)N; g.kchunk = N > 0 ? (int)N : BK;
    return launch<RSQ, true, EPI_STORE>(g, 1, as_stream(stream), what);
}

extern "C" size_t tagi_fused_weight_grad_workspace_size(int64_t M, int64_t K, int64_t N) {
    if (bad_size(M) || bad_size(K) || bad_size(N)) return 0;
    return wgrad_ws_total((int)K, (int)N, (int)M);
}

extern "C" int tagi_fused_weight_grad(const float* a, const float* dmz, const float* dSz,
                                      float* grad_mw, float* grad_Sw, int64_t M, int64_t K,
                                      int64_t N, int64_t stride_am, int64_t stride_ak,
                                      int64_t stride_dm, int64_t stride_dn, int64_t stride_km,
                                      int64_t stride_kn, void* workspace, size_t workspace_bytes,
                                      void* stream) {
    const char* what = "tagi_fused_weight_grad";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (K == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(grad_mw && grad_Sw && (M == 0 || (a && dmz && dSz)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    // x[i = k, r = m] = a[m, k]
    g.x = a; g.arow = plain_rows(stride_ak); g.ak = stride_am;
    g.u = dmz; g.v = dSz; g.brow = plain_rows(stride_dm); g.bn = stride_dn;
    g.o0 = grad_mw; g.o1 = grad_Sw; g.orow = plain_rows(stride_km); g.on = stride_kn;
    g.N = (int)N; g.Kr = (int)M;
    return run_wgrad(g, (int)K, workspace, workspace_bytes, false, as_stream(stream), what);
}

extern "C" size_t tagi_param_grad_workspace_size(int64_t M, int64_t K, int64_t N, int has_bias) {
    if (bad_size(M) || bad_size(K) || bad_size(N)) return 0;
    const int Mo = (int)K + (has_bias ? 1 : 0);
    if (bias_apart(Mo, (int)N, (int)M, has_bias != 0)) {
        size_t off = 0;
        return bias_apart_bytes(Mo, (int)N, (int)M, &off);
    }
    return wgrad_ws_total(Mo, (int)N, (int)M);
}

namespace tagi {
namespace {
// The weight-gradient family with the activations given either as a (M x K,
// row stride lda: a_rows = 1, a_k = lda) or transposed (K x M: a_rows = lda,
// a_k = 1).
int param_grad(const char* what, const float* a, int64_t a_rows, int64_t a_k, const float* dmz,
               const float* dSz, int64_t d_div, int64_t d_outer, int64_t d_stride,
               int64_t d_nstride, int64_t M, int64_t K, int64_t N, int has_bias, int mode,
               float* mw, float* Sw, float* mb, float* Sb, float* out_m, float* out_S,
               float* out_mb, float* out_Sb, float cap_factor, void* workspace,
               size_t workspace_bytes, void* stream, const double* bias_sums = nullptr) {
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    TAGI_REQUIRE(!bias_sums || has_bias, TAGI_E_BAD_ARG, "%s: bias sums without a bias", what);
    TAGI_REQUIRE(M == 0 || (a && dmz && dSz), TAGI_E_BAD_ARG, "%s: null input", what);
    if ((K + (has_bias ? 1 : 0)) == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(mode >= TAGI_WGRAD_SUMS && mode <= TAGI_WGRAD_UPDATE, TAGI_E_BAD_ARG,
                 "%s: bad mode %d", what, mode);
    if (mode == TAGI_WGRAD_SUMS)
        TAGI_REQUIRE(out_m && out_S, TAGI_E_BAD_ARG, "%s: sums need out_m/out_S", what);
    if (mode != TAGI_WGRAD_SUMS) {
        TAGI_REQUIRE(Sw && (!has_bias || Sb), TAGI_E_BAD_ARG, "%s: null variances", what);
        TAGI_REQUIRE(cap_factor > 0.f, TAGI_E_BAD_ARG, "%s: cap_factor must be > 0", what);
    }
    if (mode == TAGI_WGRAD_DELTAS)
        TAGI_REQUIRE(out_m && out_S && (!has_bias || (out_mb && out_Sb)), TAGI_E_BAD_ARG,
                     "%s: deltas need output buffers", what);
    if (mode == TAGI_WGRAD_UPDATE)
        TAGI_REQUIRE(mw && (!has_bias || mb), TAGI_E_BAD_ARG, "%s: null means", what);
    GemmArgs g = blank();
    g.x = a; g.arow = plain_rows(a_rows); g.ak = a_k;
    g.ones_row = has_bias ? (int)K : -1;
    g.u = dmz; g.v = dSz; g.brow = RowMap{d_div, d_outer, d_stride}; g.bn = d_nstride;
    g.N = (int)N; g.Kr = (int)M;
    g.pe = ParamEpi{mode, (int)K, (int)N, mw, Sw, mb, Sb, out_m, out_S, out_mb, out_Sb,
                    cap_factor};
    return run_wgrad(g, (int)K + (has_bias ? 1 : 0), workspace, workspace_bytes, true,
                     as_stream(stream), what, bias_sums);
}
}  // namespace
}  // namespace tagi

extern "C" int tagi_param_grad(const float* a, int64_t lda, const float* dmz, const float* dSz,
                               int64_t d_div, int64_t d_outer, int64_t d_stride,
                               int64_t d_nstride, int64_t M, int64_t K, int64_t N, int has_bias,
                               int mode, float* mw, float* Sw, float* mb, float* Sb, float* out_m,
                               float* out_S, float* out_mb, float* out_Sb, float cap_factor,
                               void* workspace, size_t workspace_bytes, void* stream) {
    return param_grad("tagi_param_grad", a, 1, lda, dmz, dSz, d_div, d_outer, d_stride, d_nstride,
                      M, K, N, has_bias, mode, mw, Sw, mb, Sb, out_m, out_S, out_mb, out_Sb,
                      cap_factor, workspace, workspace_bytes, stream);
}

extern "C" int tagi_param_grad_t(const float* at, int64_t ldat, const float* dmz, const float* dSz,
                                 int64_t d_div, int64_t d_outer, int64_t d_stride,
                                 int64_t d_nstride, int64_t M, int64_t K, int64_t N, int has_bias,
                                 int mode, float* mw, float* Sw, float* mb, float* Sb,
                                 float* out_m, float* out_S, float* out_mb, float* out_Sb,
                                 float cap_factor, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    return param_grad("tagi_param_grad_t", at, ldat, 1, dmz, dSz, d_div, d_outer, d_stride,
                      d_nstride, M, K, N, has_bias, mode, mw, Sw, mb, Sb, out_m, out_S, out_mb,
                      out_Sb, cap_factor, workspace, workspace_bytes, stream);
}

extern "C" int tagi_param_grad_bias_given(const float* a, int64_t lda, int transposed,
                                          const float* dmz, const float* dSz, int64_t d_div,
                                          int64_t d_outer, int64_t d_stride, int64_t d_nstride,
                                          int64_t M, int64_t K, int64_t N,
                                          const double* bias_sums, int mode, float* mw,
                                          float* Sw, float* mb, float* Sb, float* out_m,
                                          float* out_S, float* out_mb, float* out_Sb,
                                          float cap_factor, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    const char* what = "tagi_param_grad_bias_given";
    TAGI_REQUIRE(bias_sums != nullptr, TAGI_E_BAD_ARG, "%s: null bias sums", what);
    return transposed
               ? param_grad(what, a, lda, 1, dmz, dSz, d_div, d_outer, d_stride, d_nstride, M, K,
                            N, 1, mode, mw, Sw, mb, Sb, out_m, out_S, out_mb, out_Sb, cap_factor,
                            workspace, workspace_bytes, stream, bias_sums)
               : param_grad(what, a, 1, lda, dmz, dSz, d_div, d_outer, d_stride, d_nstride, M, K,
                            N, 1, mode, mw, Sw, mb, Sb, out_m, out_S, out_mb, out_Sb, cap_factor,
                            workspace, workspace_bytes, stream, bias_sums);
}

extern "C" int tagi_apply_param_sums(const float* g_m, const float* g_S, int64_t K, int64_t N,
                                     int has_bias, float* mw, float* Sw, float* mb, float* Sb,
                                     float cap_factor, void* stream) {
    const char* what = "tagi_apply_param_sums";
    TAGI_REQUIRE(!bad_size(K) && !bad_size(N), TAGI_E_BAD_ARG, "%s: bad sizes", what);
    TAGI_REQUIRE(g_m && g_S && mw && Sw && (!has_bias || (mb && Sb)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    TAGI_REQUIRE(cap_factor > 0.f, TAGI_E_BAD_ARG, "%s: cap_factor must be > 0", what);
    ParamEpi p{TAGI_WGRAD_UPDATE, (int)K, (int)N, mw, Sw, mb, Sb, nullptr, nullptr, nullptr,
               nullptr, cap_factor};
    const int64_t total = (K + (has_bias ? 1 : 0)) * N;
    if (total == 0) return TAGI_OK;
    apply_sums_kernel<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(g_m, g_S, p, total);
    return check_launch(what);
}

extern "C" int tagi_bmm_tagi_var(const float* mu_a, const float* var_a, const float* mu_b,
                                 const float* var_b, float* mean, float* var, int64_t batch,
                                 int64_t M, int64_t L, int64_t K, int64_t sa_n, int64_t sa_m,
                                 int64_t sa_k, int64_t sb_n, int64_t sb_k, int64_t sb_l,
                                 int64_t so_n, int64_t so_m, int64_t so_l, float scale,
                                 float scale_sq, void* stream) {
    const char* what = "tagi_bmm_tagi_var";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(L) && !bad_size(K) && batch >= 0 && batch <= 65535,
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (batch == 0 || M == 0 || L == 0) return TAGI_OK;
    TAGI_REQUIRE(var && (K == 0 || (mu_a && var_a && mu_b && var_b)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = mu_a; g.y = var_a; g.arow = plain_rows(sa_m); g.ak = sa_k; g.a_bs = sa_n;
    g.u = mu_b; g.v = var_b; g.brow = plain_rows(sb_k); g.bn = sb_l; g.b_bs = sb_n;
    g.o0 = mean; g.o1 = var; g.orow = plain_rows(so_m); g.on = so_l; g.o_bs = so_n;
    g.scale0 = scale; g.scale1 = scale_sq;
    g.M = (int)M; g.N = (int)L; g.Kr = (int)K; g.kchunk = K > 0 ? (int)K : BK;
    if (mean) return launch<FULL, true, EPI_STORE>(g, (int)batch, as_stream(stream), what);
    return launch<FULL, false, EPI_STORE>(g, (int)batch, as_stream(stream), what);
}

extern "C" int tagi_bmm_shared_right(const float* a_mean, const float* a_var, const float* b,
                                     float* mean, float* var, int64_t batch, int64_t M, int64_t L,
                                     int64_t K, int64_t sa_n, int64_t sa_m, int64_t sa_k,
                                     int64_t sb_n, int64_t sb_k, int64_t sb_l, int64_t so_n,
                                     int64_t so_m, int64_t so_l, float scale, void* stream) {
    const char* what = "tagi_bmm_shared_right";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(L) && !bad_size(K) && batch >= 0 && batch <= 65535,
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (batch == 0 || M == 0 || L == 0) return TAGI_OK;
    TAGI_REQUIRE(mean && var && (K == 0 || (a_mean && a_var && b)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = a_mean; g.y = a_var; g.arow = plain_rows(sa_m); g.ak = sa_k; g.a_bs = sa_n;
    g.u = b; g.brow = plain_rows(sb_k); g.bn = sb_l; g.b_bs = sb_n;
    g.o0 = mean; g.o1 = var; g.orow = plain_rows(so_m); g.on = so_l; g.o_bs = so_n;
    g.scale0 = scale; g.scale1 = scale * scale;
    g.M = (int)M; g.N = (int)L; g.Kr = (int)K; g.kchunk = K > 0 ? (int)K : BK;
    return launch<RSQ, true, EPI_STORE>(g, (int)batch, as_stream(stream), what);
}

extern "C" int tagi_bmm_shared_left(const float* a, const float* b_mean, const float* b_var,
                                    float* mean, float* var, int64_t batch, int64_t M, int64_t L,
                                    int64_t K, int64_t sa_n, int64_t sa_m, int64_t sa_k,
                                    int64_t sb_n, int64_t sb_k, int64_t sb_l, int64_t so_n,
                                    int64_t so_m, int64_t so_l, float scale, void* stream) {
    const char* what = "tagi_bmm_shared_left";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(L) && !bad_size(K) && batch >= 0 && batch <= 65535,
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    if (batch == 0 || M == 0 || L == 0) return TAGI_OK;
    TAGI_REQUIRE(mean && var && (K == 0 || (a && b_mean && b_var)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    GemmArgs g = blank();
    g.x = a; g.arow = plain_rows(sa_m); g.ak = sa_k; g.a_bs = sa_n;
    g.u = b_mean; g.v = b_var; g.brow = plain_rows(sb_k); g.bn = sb_l; g.b_bs = sb_n;
    g.o0 = mean; g.o1 = var; g.orow = plain_rows(so_m); g.on = so_l; g.o_bs = so_n;
    g.scale0 = scale; g.scale1 = scale * scale;
    g.M = (int)M; g.N = (int)L; g.Kr = (int)K; g.kchunk = K > 0 ? (int)K : BK;
    int bn = tc_pick(LSQ, g.M, g.N, g.Kr, (int)batch);
    // Narrow tiles (<= 64 columns) stage A one row per thread in tensor memory,
    // which needs each row's reduction elements contiguous; an A read down its
    // columns (a transposed view, e.g. the attention scores in the value deltas)
    // goes through 128-column tiles, whose producers stage MN-major A.
    if (bn > 0 && bn <= 64 && sa_k != 1) bn = 128;
    return launch<LSQ, true, EPI_STORE>(g, (int)batch, as_stream(stream), what, bn);
}

// ---- weight sums without a caller workspace ---------------------------------
// The split-reduction partials of tagi_fused_weight_grad_static live in this
// array of the device image (one copy per GPU that loads the library). Host code
// must not pass `g_static_scratch` itself to a kernel: on the host the name
// denotes a stand-in, not the device address. The address is looked up once per
// device with that device current and cached.
namespace tagi {
namespace {

constexpr size_t kStaticScratchBytes = TAGI_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float* g_static_addr[kMaxDevices] = {};

int static_scratch_address(float** out, const char* what) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        set_error("%s: no usable current device (%s)", what, cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            set_error("%s: cudaGetSymbolAddress failed on device %d (%s)", what, dev,
                      cudaGetErrorString(e));
            return TAGI_E_LAUNCH;
        }
        g_static_addr[dev] = static_cast<float*>(p);
    }
    *out = g_static_addr[dev];
    return TAGI_OK;
}

}  // namespace
}  // namespace tagi

extern "C" int tagi_fused_weight_grad_static(const float* a, const float* dmz, const float* dSz,
                                             float* grad_mw, float* grad_Sw, int64_t M,
                                             int64_t K, int64_t N, int64_t stride_am,
                                             int64_t stride_ak, int64_t stride_dm,
                                             int64_t stride_dn, int64_t stride_km,
                                             int64_t stride_kn, void* stream) {
    const char* what = "tagi_fused_weight_grad_static";
    TAGI_REQUIRE(!bad_size(M) && !bad_size(N) && !bad_size(K), TAGI_E_BAD_ARG, "%s: bad sizes",
                 what);
    if (K == 0 || N == 0) return TAGI_OK;
    TAGI_REQUIRE(grad_mw && grad_Sw && (M == 0 || (a && dmz && dSz)), TAGI_E_BAD_ARG,
                 "%s: null pointer", what);
    const size_t need = wgrad_ws_bytes((int)K, (int)N, (int)M);
    TAGI_REQUIRE(need <= kStaticScratchBytes, TAGI_E_WORKSPACE,
                 "%s: this shape needs %zu bytes of scratch, more than the library's static "
                 "%zu-byte array; use tagi_fused_weight_grad with a workspace",
                 what, need, kStaticScratchBytes);
    float* scratch = nullptr;
    if (need > 0) {
        const int rc = static_scratch_address(&scratch, what);
        if (rc) return rc;
    }
    GemmArgs g = blank();
    g.x = a; g.arow = plain_rows(stride_ak); g.ak = stride_am;
    g.u = dmz; g.v = dSz; g.brow = plain_rows(stride_dm); g.bn = stride_dn;
    g.o0 = grad_mw; g.o1 = grad_Sw; g.orow = plain_rows(stride_km); g.on = stride_kn;
    g.N = (int)N; g.Kr = (int)M;
    return run_wgrad(g, (int)K, scratch, need > 0 ? kStaticScratchBytes : 0, false,
                     as_stream(stream), what);
}
