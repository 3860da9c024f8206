// Moment contractions on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// One CTA computes a 128 x BN output tile of both accumulators (mean, variance)
// of a moment contraction (see moment_gemm.cuh for the three variance forms).
// Accumulators live in tensor memory (2*BN fp32 columns). Precision is 3xTF32:
// every fp32 operand v is split into hi = tf32(v) and lo = tf32(v - hi), both
// rounded to nearest so that the tensor core sees exact tf32 values, and each
// product a*b is formed as hi*hi + hi*lo + lo*hi, dropping lo*lo (about 2^-22
// relative; the split-precision scheme of Ootomo & Yokota). Squares and mu^2 + var are formed
// in fp32 first, as the reference does, and then split.
//
// Warp roles (672 threads):
//   warps 0-7   A producers: two threads per output row, 4 reduction elements
//               each per stage; stage raw x (and y) from any row-split layout
//               through a cp.async ring, form the split operand tiles and store
//               them in the canonical no-swizzle K-major layout (8x16-byte core
//               matrices).
//   warps 8-15  B producers: the same for u (and v), one row per output column.
//   warp 16     allocates tensor memory; lane 0 issues the tcgen05.mma
//               instructions and commits them to the stage's "empty" barrier.
//   warps 17-20 accumulator warps (TMEM lane quarter warp % 4): the tensor
//              core's fp32 accumulation truncates, so products are accumulated
//              in tensor memory for kChunk stages only; these warps fold each
//              chunk into a running total with round-to-nearest adds and run the
//              epilogue from the last fold.
// Stages form a ring of STAGES shared-memory buffers guarded by mbarriers.
// Every wait is bounded: on timeout the CTA records an error word
// (tagi_device_status), stops issuing work, waits (bounded) for its MMAs and
// frees its tensor memory before returning.
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "moment_gemm.cuh"

namespace tagi {

__device__ int g_device_error = 0;  // 0 = ok, else the code of the first timeout

namespace {

constexpr int kStages = 4;
constexpr int kBK = 8;  // tf32 elements per MMA along the reduction
constexpr int kThreads = 672;  // 21 warps
constexpr int kChunk = 16;     // stages accumulated in tensor memory before a fold
constexpr int kRawStages = 4;  // depth of the cp.async ring of raw operand rows
constexpr int kRawSlot = 2 * 256 * 32;  // two operands x 256 producer rows x 8 fp32
enum { kScalar = 0, kRowK = 1, kKRow = 2 };
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false if the CTA aborted or timed out.
__device__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(bar, parity)) return true;
        if ((it & 255u) == 255u) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kTimeoutNs) {
                *abort_flag = 1;
                atomicCAS(&g_device_error, 0, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
// 4-byte copy; when `ok` is false nothing is read and the destination is zeroed.
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(ok ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive columns of this warp's 32 lanes; completes at tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

template <int EPI, bool MEAN>
__device__ __forceinline__ void store_out(const GemmArgs& g, int row, int col, int64_t ro,
                                          int split, float a0, float a1) {
    if (EPI == EPI_STORE) {
        const int64_t o = ro + static_cast<int64_t>(col) * g.on;
        if (MEAN && g.o0) g.o0[o] = g.scale0 * a0 + (g.bias0 ? g.bias0[col] : 0.f);
        g.o1[o] = g.scale1 * a1 + (g.bias1 ? g.bias1[col] : 0.f);
    } else if (EPI == EPI_PARTIAL) {
        const int64_t mn = static_cast<int64_t>(g.M) * g.N;
        const int64_t o = static_cast<int64_t>(row) * g.N + col;
        g.ws[(2 * split) * mn + o] = a0;
        g.ws[(2 * split + 1) * mn + o] = a1;
    } else {
        param_epilogue(row, col, a0, a1, g.pe);
    }
}

// Shared-memory matrix descriptor: no swizzle, K-major, core matrices of 8 rows
// x 16 bytes; the two 16-byte halves of a row's 8 tf32 values are 128 bytes
// apart (leading byte offset) and consecutive 8-row groups 256 bytes apart
// (stride byte offset). Bit 46 carries the descriptor version of sm_100.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
           (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor: fp32 accumulate, tf32 A and B, both K-major, M=128.
__host__ __device__ constexpr uint32_t instr_desc(int bn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(bn >> 3) << 17) |
           (static_cast<uint32_t>(128 >> 4) << 24);
}

// Nearest tf32 value (ties away from zero): add half a tf32 ulp to the
// magnitude bits and clear the 13 bits that tf32 drops.
__device__ __forceinline__ float tf32_rna(float v) {
    return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// Byte offset of (row, k-half) inside a K-major no-swizzle tile of 8-element rows.
__device__ __forceinline__ uint32_t tile_off(int row, int half) {
    return static_cast<uint32_t>((row >> 3) * 256 + half * 128 + (row & 7) * 16);
}

// Split four fp32 values into tf32 hi/lo parts and store them (16 bytes each).
__device__ __forceinline__ void st_split4(char* tile_hi, char* tile_lo, uint32_t off,
                                          const float (&v)[4]) {
    float4 hi, lo;
    hi.x = tf32_rna(v[0]); lo.x = tf32_rna(v[0] - hi.x);
    hi.y = tf32_rna(v[1]); lo.y = tf32_rna(v[1] - hi.y);
    hi.z = tf32_rna(v[2]); lo.z = tf32_rna(v[2] - hi.z);
    hi.w = tf32_rna(v[3]); lo.w = tf32_rna(v[3] - hi.w);
    *reinterpret_cast<float4*>(tile_hi + off) = hi;
    *reinterpret_cast<float4*>(tile_lo + off) = lo;
}

template <int VM>
struct TcTiles {
    static constexpr int na = (VM == FULL) ? 6 : 4;
    static constexpr int nb = (VM == FULL) ? 6 : 4;
};

// (accumulator, A tile, B tile) of every MMA of one stage, packed as 4-bit
// fields (entry i at bits [4i, 4i+4)).
template <int VM>
struct TcPlan;
template <>
struct TcPlan<FULL> {  // A: x, x^2, y ; B: u, v, u^2+v   (hi, lo pairs)
    static constexpr int n = 9;
    static constexpr unsigned long long acc = 0x111111000ull;
    static constexpr unsigned long long a = 0x544322100ull;
    static constexpr unsigned long long b = 0x454232010ull;
};
template <>
struct TcPlan<RSQ> {  // A: x, y ; B: u, u^2
    static constexpr int n = 6;
    static constexpr unsigned long long acc = 0x111000ull;
    static constexpr unsigned long long a = 0x322100ull;
    static constexpr unsigned long long b = 0x232010ull;
};
template <>
struct TcPlan<LSQ> {  // A: x, x^2 ; B: u, v
    static constexpr int n = 6;
    static constexpr unsigned long long acc = 0x111000ull;
    static constexpr unsigned long long a = 0x322100ull;
    static constexpr unsigned long long b = 0x232010ull;
};

__host__ __device__ constexpr int field(unsigned long long packed, int i) {
    return static_cast<int>((packed >> (4 * i)) & 0xFull);
}

template <int VM, int BN>
constexpr int stage_bytes() {
    return TcTiles<VM>::na * 128 * 32 + TcTiles<VM>::nb * BN * 32;
}

// Operand stages that fit next to the raw ring in 227 KB (at most kStages).
template <int VM, int BN>
constexpr int op_stages() {
    return (220 * 1024 - kRawStages * kRawSlot) / stage_bytes<VM, BN>() < kStages
               ? (220 * 1024 - kRawStages * kRawSlot) / stage_bytes<VM, BN>()
               : kStages;
}

template <int VM, int BN>
constexpr int smem_bytes() {
    return op_stages<VM, BN>() * stage_bytes<VM, BN>() + kRawStages * kRawSlot + 1024;
}


// Number of chunk accumulators P (double-buffered when tensor memory allows).
template <int BN>
constexpr int num_p() {
    return 6 * BN <= 512 ? 2 : 1;
}

template <int BN>
constexpr int tmem_cols() {
    return (num_p<BN>() + 1) * 2 * BN <= 128 ? 128 : ((num_p<BN>() + 1) * 2 * BN <= 256 ? 256 : 512);
}

template <int VM, bool MEAN, int EPI, int BN>
__global__ void __launch_bounds__(kThreads, 1) moment_tc_kernel(const GemmArgs g) {
    using T = TcTiles<VM>;
    using P = TcPlan<VM>;
    constexpr int A_TILE = 128 * 32, B_TILE = BN * 32;
    constexpr int STAGE = stage_bytes<VM, BN>();
    constexpr int NP = num_p<BN>();
    constexpr int COLS = tmem_cols<BN>();
    constexpr int OPS = op_stages<VM, BN>();
    extern __shared__ __align__(1024) char smem[];
    char* raw = smem + OPS * STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(raw + kRawStages * kRawSlot);
    uint64_t* empty = full + kStages;
    uint64_t* chunk_full = empty + kStages;   // [NP]: MMA -> accumulator warps
    uint64_t* chunk_empty = chunk_full + 2;   // [NP]: accumulator warps -> MMA
    uint64_t* done = chunk_empty + 2;         // all MMAs complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128;
    const int batch = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
    const int kbeg = split * g.kchunk;
    const int kend = min(g.Kr, kbeg + g.kchunk);
    const int niter = kend > kbeg ? (kend - kbeg + kBK - 1) / kBK : 0;
    const int nchunks = (niter + kChunk - 1) / kChunk;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 512);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&chunk_full[b], 1);
            mbar_init(&chunk_empty[b], 128);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async();
    }
    if (warp == 16) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // columns: P buffer b at [2*BN*b, 2*BN*(b+1)), running total T after them;
    // within each, the mean accumulator then the variance accumulator.
    const uint32_t tcol_total = 2 * BN * NP;

    if (warp < 16) {
        // ---------------------------------------------------------------- producers
        // Two threads per tile row: `half` selects reduction elements 0-3 or 4-7.
        const bool is_a = warp < 8;
        const int side_tid = is_a ? tid : tid - 256;
        const int r = side_tid & 127, half = side_tid >> 7;
        const bool active = is_a ? true : (r < BN);
        int idx;
        bool valid, one = false;
        int64_t base = 0;
        const float *p0, *p1;
        if (is_a) {
            idx = m0 + r;
            valid = idx < g.M;
            one = (idx == g.ones_row);
            base = (valid && !one) ? g.arow.off(idx) : 0;
            p0 = g.x + batch * g.a_bs;
            p1 = (VM == LSQ) ? nullptr : g.y + batch * g.a_bs;
        } else {
            idx = n0 + r;
            valid = active && idx < g.N;
            base = valid ? static_cast<int64_t>(idx) * g.bn : 0;
            p0 = g.u + batch * g.b_bs;
            p1 = (VM == RSQ) ? nullptr : g.v + batch * g.b_bs;
        }
        const bool has1 = (p1 != nullptr);
        // Staging modes of this side's operands (uniform over the side):
        //  kRowK   each row's reduction values are contiguous and 16-byte aligned:
        //          a thread copies its own 4-element half row as one 16-byte chunk
        //          ([row][8] layout);
        //  kKRow   4 consecutive rows are contiguous and aligned for every reduction
        //          index: the side's 256 threads copy one 16-byte row chunk each into a
        //          [k][128] layout and read it transposed after a named barrier;
        //  kScalar element-wise 4-byte copies of the thread's own half row.
        // Out-of-range elements are zero-filled; chunks that straddle a tile edge or
        // the bias row fall back to element-wise copies.
        const uintptr_t align_bits = (reinterpret_cast<uintptr_t>(p0) |
                                      (has1 ? reinterpret_cast<uintptr_t>(p1) : 0)) & 15;
        int mode = kScalar;
        if (is_a) {
            const RowMap& m = g.arow;
            const bool rows4 = (m.div <= 0) ? (m.stride % 4 == 0)
                                            : (m.stride % 4 == 0 && m.outer % 4 == 0);
            if (align_bits == 0 && g.ak == 1 && rows4) {
                mode = kRowK;
            } else if (align_bits == 0 && m.stride == 1 && g.ak % 4 == 0 &&
                       (m.div <= 0 || (m.div % 4 == 0 && m.outer % 4 == 0))) {
                mode = kKRow;
            }
        } else {
            const RowMap& m = g.brow;
            if (align_bits == 0 && m.stride == 1 && g.bn % 4 == 0 &&
                (m.div <= 0 || (m.div % 8 == 0 && m.outer % 4 == 0))) {
                mode = kRowK;
            } else if (align_bits == 0 && g.bn == 1 &&
                       ((m.div <= 0) ? (m.stride % 4 == 0)
                                     : (m.stride % 4 == 0 && m.outer % 4 == 0))) {
                mode = kKRow;
            }
        }
        const int side_rows = is_a ? g.M : g.N;
        const int side_row0 = is_a ? m0 : n0;
        // region of (slot, operand) for this side: 128 rows x 8 fp32
        auto region = [&](int slot, int o) -> char* {
            return raw + slot * kRawSlot + ((is_a ? 0 : 2) + o) * 4096;
        };
        // global offset of (row, k) for this side, valid row and k < kend assumed
        auto goff = [&](int rrow, int k) -> int64_t {
            return is_a ? g.arow.off(rrow) + static_cast<int64_t>(k) * g.ak
                        : static_cast<int64_t>(rrow) * g.bn + g.brow.off(k);
        };
        auto row_ok = [&](int rrow) -> bool {
            return rrow < side_rows && !(is_a && rrow == g.ones_row);
        };
        auto issue = [&](int it) {
            if (it >= niter) return;
            const int k0 = kbeg + it * kBK;
            const int slot = it % kRawStages;
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                if (o == 1 && !has1) break;
                const float* src = o ? p1 : p0;
                char* reg = region(slot, o);
                if (mode == kKRow) {
                    const int c = side_tid;  // chunk: k = c / 32, rows 4*(c % 32) .. +3
                    const int k = k0 + c / 32, rg = c % 32;
                    const int rrow = side_row0 + 4 * rg;
                    char* dst = reg + (c / 32) * 512 + rg * 16;
                    if (4 * rg < (is_a ? 128 : BN)) {
                        if (k < kend && rrow + 3 < side_rows &&
                            !(is_a && g.ones_row >= rrow && g.ones_row <= rrow + 3)) {
                            cp_async16(dst, src + goff(rrow, k));
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const bool ok = k < kend && row_ok(rrow + q);
                                cp_async4(dst + 4 * q, ok ? src + goff(rrow + q, k) : src, ok);
                            }
                        }
                    }
                } else {
                    if (!valid || one) continue;
                    const int kh = k0 + 4 * half;
                    char* dst = reg + r * 32 + half * 16;
                    if (mode == kRowK && kh + 4 <= kend) {
                        cp_async16(dst, src + goff(idx, kh));
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int k = kh + j;
                            const bool ok = k < kend;
                            cp_async4(dst + 4 * j, ok ? src + goff(idx, k) : src, ok);
                        }
                    }
                }
            }
        };
        auto fetch = [&](int it, float (&v0)[4], float (&v1)[4]) {
            const int kh = kbeg + it * kBK + 4 * half;
            if (!valid) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v0[j] = v1[j] = 0.f;
                return;
            }
            if (one) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v0[j] = (kh + j < kend) ? 1.f : 0.f;
                    v1[j] = 0.f;
                }
                return;
            }
            const int slot = it % kRawStages;
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                float* v = o ? v1 : v0;
                if (o == 1 && !has1) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = 0.f;
                    break;
                }
                const char* reg = region(slot, o);
                if (mode == kKRow) {
                    const float* f = reinterpret_cast<const float*>(reg);
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = f[(4 * half + j) * 128 + r];
                } else {
                    const float4 x = *reinterpret_cast<const float4*>(reg + r * 32 + half * 16);
                    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
                }
            }
        };

        auto produce = [&](int it, const float (&v0)[4], const float (&v1)[4]) -> bool {
            const int s = it % OPS;
            if (it >= OPS && !mbar_wait(&empty[s], ((it / OPS) & 1) ^ 1, abort_flag, 1))
                return false;
            if (active) {
                char* st = smem + s * STAGE;
                const uint32_t off = tile_off(r, half);
                float sq[4];
                if (is_a) {
                    char* A = st;
                    st_split4(A + 0 * A_TILE, A + 1 * A_TILE, off, v0);
                    if (VM == FULL || VM == LSQ) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) sq[j] = v0[j] * v0[j];
                        st_split4(A + 2 * A_TILE, A + 3 * A_TILE, off, sq);
                    }
                    if (VM == FULL) st_split4(A + 4 * A_TILE, A + 5 * A_TILE, off, v1);
                    if (VM == RSQ) st_split4(A + 2 * A_TILE, A + 3 * A_TILE, off, v1);
                } else {
                    char* B = st + T::na * A_TILE;
                    st_split4(B + 0 * B_TILE, B + 1 * B_TILE, off, v0);
                    if (VM == FULL) {
                        st_split4(B + 2 * B_TILE, B + 3 * B_TILE, off, v1);
#pragma unroll
                        for (int j = 0; j < 4; ++j) sq[j] = v0[j] * v0[j] + v1[j];
                        st_split4(B + 4 * B_TILE, B + 5 * B_TILE, off, sq);
                    } else if (VM == RSQ) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) sq[j] = v0[j] * v0[j];
                        st_split4(B + 2 * B_TILE, B + 3 * B_TILE, off, sq);
                    } else {
                        st_split4(B + 2 * B_TILE, B + 3 * B_TILE, off, v1);
                    }
                }
                fence_proxy_async();
            }
            mbar_arrive(&full[s]);
            return true;
        };

        // cp.async ring: kRawStages-1 stages in flight ahead of the one transformed
        for (int i = 0; i < kRawStages - 1; ++i) {
            issue(i);
            cp_async_commit();
        }
        float v0[4], v1[4];
        // After an abort every thread keeps iterating without work, so that all
        // threads of a side still reach every named barrier.
        bool alive = true;
        for (int it = 0; it < niter; ++it) {
            cp_async_wait<kRawStages - 2>();
            // rows staged by other threads of this side: wait until all copied (and
            // until all consumed the slot that the next issue refills)
            if (mode == kKRow) named_bar_sync(is_a ? 1 : 2, 256);
            if (alive) {
                fetch(it, v0, v1);
                alive = produce(it, v0, v1);
            }
            if (alive) issue(it + kRawStages - 1);  // refills the slot consumed one iteration ago
            cp_async_commit();
        }
        cp_async_wait<0>();
    } else if (warp == 16) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issue
            constexpr uint32_t idesc = instr_desc(BN);
            const uint32_t base = smem_u32(smem);
            bool started[2] = {false, false};
            for (int it = 0; it < niter; ++it) {
                const int c = it / kChunk, b = c % NP;
                if (it % kChunk == 0) {
                    // chunk c accumulates into buffer b once the fold of chunk c-NP freed it
                    if (c >= NP && !mbar_wait(&chunk_empty[b], ((c / NP) - 1) & 1, abort_flag, 5))
                        break;
                    tc_fence_after();
                    started[0] = started[1] = false;
                }
                const int s = it % OPS;
                if (!mbar_wait(&full[s], (it / OPS) & 1, abort_flag, 2)) break;
                tc_fence_after();
                const uint32_t st = base + s * STAGE;
                const uint32_t pcol = tmem + static_cast<uint32_t>(2 * BN * b);
#pragma unroll
                for (int i = 0; i < P::n; ++i) {
                    const int acc = field(P::acc, i);
                    if (!MEAN && acc == 0) continue;
                    const uint64_t ad = smem_desc(st + field(P::a, i) * A_TILE);
                    const uint64_t bd = smem_desc(st + T::na * A_TILE + field(P::b, i) * B_TILE);
                    mma_tf32(pcol + acc * BN, ad, bd, idesc, started[acc] ? 1u : 0u);
                    started[acc] = true;
                }
                mma_commit(&empty[s]);
                if (it % kChunk == kChunk - 1 || it == niter - 1) mma_commit(&chunk_full[b]);
            }
            mma_commit(done);  // arrives once every MMA issued above has completed
        }
    } else {
        // -------------------------------------------- accumulator warps (17-20)
        // Tensor-core accumulation truncates; each chunk of kChunk stages is
        // folded into the running total with round-to-nearest fp32 adds, and the
        // last fold feeds the epilogue directly.
        const int sub = warp & 3;  // TMEM lane quarter this warp may access
        const int row = m0 + sub * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(sub * 32) << 16);
        bool ok = true;
        for (int c = 0; c < nchunks && ok; ++c) {
            const int b = c % NP;
            ok = __all_sync(0xffffffffu, mbar_wait(&chunk_full[b], (c / NP) & 1, abort_flag, 3) &&
                                             !*abort_flag);
            if (!ok) break;
            tc_fence_after();
            const bool last = (c == nchunks - 1);
            const uint32_t pcol = lane_base + static_cast<uint32_t>(2 * BN * b);
            const uint32_t tcol = lane_base + tcol_total;
            const int64_t ro =
                (EPI == EPI_STORE && row < g.M) ? g.orow.off(row) + batch * g.o_bs : 0;
            // Intermediate folds: T += P, 16 columns at a time, the P and T loads of a
            // column block issued together before one wait.
            if (!last) {
#pragma unroll 1
                for (int c0 = 0; c0 < 2 * BN; c0 += 16) {
                    if (!MEAN && c0 < BN) continue;
                    uint32_t pr[16], tr[16];
                    tmem_ld16_async(pcol + c0, pr);
                    if (c > 0) tmem_ld16_async(tcol + c0, tr);
                    tmem_wait_ld();
                    float tv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        tv[j] = c > 0 ? __uint_as_float(tr[j]) + __uint_as_float(pr[j])
                                      : __uint_as_float(pr[j]);
                    tmem_st16(tcol + c0, tv);
                }
            } else {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float pm[16], pv[16], tm[16], tv[16];
                    if (MEAN) tmem_ld16(pcol + c0, pm);
                    tmem_ld16(pcol + BN + c0, pv);
                    if (c > 0) {
                        if (MEAN) tmem_ld16(tcol + c0, tm);
                        tmem_ld16(tcol + BN + c0, tv);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        tm[j] = MEAN ? (c > 0 ? tm[j] + pm[j] : pm[j]) : 0.f;
                        tv[j] = c > 0 ? tv[j] + pv[j] : pv[j];
                    }
                    if (row >= g.M) continue;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = n0 + c0 + j;
                        if (col >= g.N) continue;
                        store_out<EPI, MEAN>(g, row, col, ro, split, tm[j], tv[j]);
                    }
                }
            }
            if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&chunk_empty[b]);
        }
        if (nchunks == 0 && row < g.M) {
            // empty reduction: outputs are the biases (or zero sums)
            const int64_t ro = (EPI == EPI_STORE) ? g.orow.off(row) + batch * g.o_bs : 0;
            for (int col = n0; col < min(n0 + BN, g.N); ++col)
                store_out<EPI, MEAN>(g, row, col, ro, split, 0.f, 0.f);
        }
    }

    if (warp == 16) {
        // the MMAs of this CTA must be complete before their memory is released
        if (!mbar_try(done, 0)) mbar_wait(done, 0, abort_flag, 4);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 16) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(COLS));
    }
}

bool tc_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = std::getenv("TAGI_B200_TC");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

template <int VM, bool MEAN, int EPI, int BN>
int launch_tc(const GemmArgs& g, int batch, cudaStream_t st, const char* what) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    constexpr int smem = smem_bytes<VM, BN>();
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(moment_tc_kernel<VM, MEAN, EPI, BN>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr_err != cudaSuccess) {
        set_error("%s: cannot reserve %d bytes of shared memory (%s)", what, smem,
                  cudaGetErrorString(attr_err));
        return TAGI_E_LAUNCH;
    }
    dim3 grid((g.N + BN - 1) / BN, (g.M + 127) / 128, batch * g.splits);
    TAGI_REQUIRE(grid.y <= 65535 && grid.z <= 65535, TAGI_E_UNSUPPORTED, "%s: grid too large",
                 what);
    moment_tc_kernel<VM, MEAN, EPI, BN><<<grid, kThreads, smem, st>>>(g);
    return check_launch(what);
}

template <int VM, bool MEAN, int EPI>
int launch_bn(const GemmArgs& g, int bn, int batch, cudaStream_t st, const char* what) {
    switch (bn) {
        case 32: return launch_tc<VM, MEAN, EPI, 32>(g, batch, st, what);
        case 64: return launch_tc<VM, MEAN, EPI, 64>(g, batch, st, what);
        default: return launch_tc<VM, MEAN, EPI, 128>(g, batch, st, what);
    }
}

}  // namespace

int tc_pick(int vm, int M, int N, int Kr, int batch) {
    (void)vm;
    (void)batch;
    if (!tc_enabled()) return 0;
    if (M < 64 || N < 16 || Kr < 32) return 0;
    if (static_cast<double>(M) * N * Kr < 4.0e6) return 0;
    if (N <= 32) return 32;
    if (N <= 64) return 64;
    return 128;
}

int tc_launch(const GemmArgs& g, int vm, bool mean, int epi, int bn, int batch, cudaStream_t st,
              const char* what) {
    if (g.M == 0 || g.N == 0) return TAGI_OK;
    if (vm == FULL) {
        if (epi != EPI_STORE) return TAGI_E_UNSUPPORTED;
        return mean ? launch_bn<FULL, true, EPI_STORE>(g, bn, batch, st, what)
                    : launch_bn<FULL, false, EPI_STORE>(g, bn, batch, st, what);
    }
    if (vm == RSQ) {
        if (epi != EPI_STORE || !mean) return TAGI_E_UNSUPPORTED;
        return launch_bn<RSQ, true, EPI_STORE>(g, bn, batch, st, what);
    }
    if (!mean) return TAGI_E_UNSUPPORTED;
    switch (epi) {
        case EPI_STORE: return launch_bn<LSQ, true, EPI_STORE>(g, bn, batch, st, what);
        case EPI_PARTIAL: return launch_bn<LSQ, true, EPI_PARTIAL>(g, bn, batch, st, what);
        default: return launch_bn<LSQ, true, EPI_PARAM>(g, bn, batch, st, what);
    }
}

}  // namespace tagi

extern "C" int tagi_device_status(int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, tagi::g_device_error, sizeof(int));
    if (e != cudaSuccess) {
        cudaGetLastError();
        tagi::set_error("tagi_device_status: %s", cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    if (reset && v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(tagi::g_device_error, &zero, sizeof(int));
    }
    return v;
}
