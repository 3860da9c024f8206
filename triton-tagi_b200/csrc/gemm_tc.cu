// Moment contractions on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Tiles. A cluster of two CTAs computes a 256 x BN tile of both accumulators
// (mean, variance) of a moment contraction (moment_gemm.cuh has the three
// variance forms) with 2-SM MMAs (tcgen05.mma.cta_group::2, M = 256). Each CTA
// stages its own 128 rows of the A operands and half of the B operands (BN/2
// rows) in shared memory and keeps the accumulator rows of its half in its own
// tensor memory; the pair's tensor cores share B. Per 128 x 128 x 8 product an
// SM then reads 6 KB of operands from shared memory instead of 8 KB, and that is
// what lets the MMAs run at the tensor pipe's rate: a single-CTA 128 x 128 tile
// is bound by shared-memory bandwidth at about three quarters of it.
//
// Precision is 3xTF32: every fp32 operand v is split into hi = tf32(v) and
// lo = tf32(v - hi), both rounded to nearest so that the tensor core sees exact
// tf32 values, and each product a*b is formed as hi*hi + hi*lo + lo*hi, dropping
// lo*lo (about 2^-22 relative; the split-precision scheme of Ootomo & Yokota).
// Squares and mu^2 + var are formed in fp32 first, as the reference does, and
// then split. The tensor core's fp32 accumulation truncates, so products are
// accumulated in tensor memory for kChunk stages only and each chunk is folded
// into a running total with round-to-nearest fp32 adds.
//
// Warp roles (per CTA):
//   warps 0-7     A producers in two groups of four; group g serves the stages
//                 of parity g and each thread one tile row. A thread loads its
//                 row's 8 reduction elements per stage from global memory
//                 straight into registers (its next stage in flight),
//                 splits them and stores the operand tiles in the canonical
//                 no-swizzle K-major layout (8-row x 16-byte core matrices).
//   next 2*BW     B producers: the same for this CTA's BN/2 rows of B.
//   MMA warp      allocates tensor memory (both CTAs); in the leader CTA
//                 (cluster rank 0) it runs the stage loop and an elected lane
//                 issues the MMAs and commits them to barriers of both CTAs
//                 (multicast commit).
//   8 acc warps   fold chunks and run the epilogue; warp w reads tensor-memory
//                 lane quarter w % 4 and one half of the columns.
// The mean and variance chunks end on staggered stages: when a chunk buffer must
// be drained before reuse, the MMA warp issues the other accumulator's products
// of the stage first and waits for the fold only then.
//
// Every wait is bounded: on timeout a CTA records an error word
// (tagi_device_status), tells its peer, stops issuing work, waits (bounded) for
// its MMAs and frees its tensor memory before returning.
#include <cuda.h>

#include <atomic>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "moment_gemm.cuh"

namespace tagi {

__device__ int g_device_error = 0;  // 0 = ok, else the code of the first timeout
// Limit of the waits that give up the tile (the producers', the MMA issuer's and
// the accumulator warps'). tagi_set_wait_limit_ns changes it so that a test can
// make those waits run out; the drains that must complete before a CTA exits
// (its own bulk copies, its MMAs) keep the fixed kTimeoutNs.
__device__ unsigned long long g_wait_limit_ns = 2000000000ull;
// Test hook: non-zero makes every launch give up its tiles at the start, as a
// wait that ran out would (the abort, drain and release path then runs).
__device__ int g_force_abort = 0;

namespace {

constexpr int kBK = 8;              // tf32 elements per MMA along the reduction
constexpr int kChunk = 16;          // stages accumulated in tensor memory before a fold
// K-blocks loaded ahead per producer thread (each group owns every other
// K-block). Two for the 64-column tiles of 64-channel convolutions was slower
// than one (measured: weight sums 1.73 -> 2.04 ms, input deltas 1.44 -> 1.63 ms
// per ResNet-18 step), so one throughout.
template <int BN>
constexpr int prefetch_depth() { return 1; }
constexpr int kMaxStages = 8;       // operand stages in shared memory
constexpr int kStageBudget = 224 * 1024;
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

// Warp layout and tensor-memory plan of a CTA for a pair tile of BN columns.
template <int BN>
struct Roles {
    static constexpr int NC = BN / 2;                  // B rows staged by each CTA
    static constexpr int BW = NC >= 32 ? NC / 32 : 1;  // B producer warps per group
    static constexpr int B_W0 = 8;
    static constexpr int MMA_W = B_W0 + 2 * BW;
    static constexpr int ACC_W0 = MMA_W + 1;
    static constexpr int WARPS = ACC_W0 + 8;
    static constexpr int THREADS = 32 * WARPS;
    static constexpr int STAGE_ARRIVALS = 2 * 2 * (4 + BW);  // producer warps of a stage: 2 groups, 2 CTAs
    // Tiles of 64 columns or fewer keep the A operand in tensor memory (TA):
    // their MMAs are bound by operand traffic in shared memory, where each
    // 256 x 64 x 8 MMA would read a 4 KB A tile per CTA; the chunk buffers then
    // take one slot per accumulator and the remaining columns hold the A stages.
    static constexpr bool TA = BN <= 64;
    static constexpr int NP = TA ? 1 : (6 * BN <= 512 ? 2 : 1);  // chunk buffers per accumulator
    static constexpr int ACC_COLS = 2 * (NP + 1) * BN;
    static constexpr int COLS = (TA || ACC_COLS > 256) ? 512 : 256;
    static constexpr uint32_t A0 = ACC_COLS;  // first tensor-memory column of the A stages (TA)
    // tensor-memory columns: chunk buffer b of accumulator q, running total of q
    static constexpr uint32_t pcol(int q, int b) { return static_cast<uint32_t>((q * NP + b) * BN); }
    static constexpr uint32_t tcol(int q) { return static_cast<uint32_t>((2 * NP + q) * BN); }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Arrive on a barrier given by its cluster shared-memory address (own or peer
// CTA), with the default release semantics at CTA scope. A cluster-scope release
// would make the arriving warp wait for all of its global loads in flight, which
// are the producers' prefetches of later stages.
__device__ __forceinline__ void arrive_cluster(uint32_t addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

// Test for completion of phase `parity` (default acquire semantics at CTA scope,
// as for the other barriers of the pair); a waiting thread is suspended (it
// takes no issue slots) until the phase completes or about kSuspendNs passed.
// (The hint is an immediate: reading it from memory in every wait slowed the
// contractions by 4 %.)
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

struct Abort {
    volatile int* flag;  // this CTA's abort word
    uint32_t peer;       // cluster address of the peer CTA's abort word
};

// Bounded wait (after a failed first test); false if the pair aborted or timed out.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, const Abort& ab,
                                            int code) {
    const unsigned long long t0 = globaltimer();
    const unsigned long long limit = *const_cast<volatile unsigned long long*>(&g_wait_limit_ns);
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (*ab.flag) return false;
        if (globaltimer() - t0 > limit) {
            *ab.flag = 1;
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(ab.peer), "r"(1) : "memory");
            atomicCAS(&g_device_error, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const Abort& ab,
                                          int code) {
    return mbar_try(bar, parity) || mbar_wait_slow(bar, parity, ab, code);
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const Abort& ab,
                                          int code) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, ab, code));
}

// Bounded wait that ignores the abort flag: for bulk copies this warp issued,
// which must land before the CTA may exit.
__device__ __noinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try(bar, parity))
        if (globaltimer() - t0 > kTimeoutNs) return false;
    return true;
}

// Arrive on a barrier of this CTA.
__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on a local barrier and add `bytes` to the transactions its phase waits for.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bulk asynchronous copy of `bytes` (a multiple of 16, both addresses 16-byte
// aligned) from global memory into this CTA's shared memory; completes as
// transactions on `bar`. No multicast: the source is this GPU's own memory and
// only the issuing CTA receives it.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Tensor-map tile copies into this CTA's shared memory (no multicast; the
// source is this GPU's own memory), completing as transactions on `bar`. The
// innermost coordinate x is a multiple of 8 fp32 elements (32 bytes).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool elect_one() {
    uint32_t p;
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}"
        : "=r"(p));
    return p != 0;
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

__device__ __forceinline__ void mma_pair_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with the A operand in tensor memory (column a_tmem of both CTAs).
__device__ __forceinline__ void mma_pair_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Stores 8 consecutive 32-bit columns of this thread's lane (one warp: 32
// lanes of its quarter) at taddr.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
        : "memory");
}

// Arrives on `bar` in both CTAs of the pair once all MMAs issued so far completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_u32(bar)),
        "h"(static_cast<unsigned short>(3))
        : "memory");
}

// 16 consecutive columns of this warp's 32 lanes; complete at tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
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
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// Shared-memory matrix descriptors (bit 46 carries the descriptor version of
// sm_100). An operand tile holds `rows` rows x 8 tf32 reduction elements
// (rows * 32 bytes) in one of two canonical layouts:
//   K-major, no swizzle: core matrices of 8 rows x 16 bytes (4 reduction
//     elements); the two halves of a row's 8 elements are 128 bytes apart
//     (leading byte offset) and consecutive 8-row groups 256 bytes apart (stride
//     byte offset): byte (row/8)*256 + (k/4)*128 + (row%8)*16 + (k%4)*4.
//   MN-major, 128-byte swizzle on a 32-byte base (the MN-major layout that tf32
//     operands accept; layout type 1): atoms of 4 reduction rows x 128 bytes
//     (32 tile rows), the 32-byte chunks of reduction row kr XOR-permuted by kr;
//     atoms along the tile rows 512 bytes apart (leading byte offset), the two
//     4-row reduction groups rows*16 bytes apart (stride byte offset). Tiles
//     start 512-byte aligned so that the address bits the swizzle reads are the
//     atom's own row index.
// The start address occupies the low 14 bits (address / 16), so descriptors of
// tiles inside one stage differ by (byte offset / 16).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, bool mn_major, int rows) {
    const uint64_t lbo = mn_major ? 512 : 128;
    const uint64_t sbo = mn_major ? static_cast<uint64_t>(rows) * 16 : 256;
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | ((lbo >> 4) << 16) | ((sbo >> 4) << 32) |
           (1ull << 46) | (mn_major ? (1ull << 61) : 0ull);
}
__device__ __forceinline__ uint32_t tile_off_k(int row, int k) {
    return static_cast<uint32_t>((row >> 3) * 256 + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4);
}
// MN-major byte offset of (row, k) for a tile of `rows` rows; rows 4j..4j+3 at
// one k are 16 contiguous bytes.
__device__ __forceinline__ uint32_t tile_off_mn(int row, int k, int rows) {
    const int mn = row & 31, kr = k & 3;
    return static_cast<uint32_t>((row >> 5) * 512 + (k >> 2) * rows * 16 + kr * 128 +
                                 (((mn >> 3) ^ kr) << 5) + (mn & 7) * 4);
}

// Instruction descriptor: fp32 accumulate, tf32 A and B, M = 256 (2-SM),
// N = bn; bits 15 and 16 select MN-major A and B.
__device__ __forceinline__ uint32_t instr_desc(int bn, bool a_mn, bool b_mn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (a_mn ? 1u << 15 : 0u) | (b_mn ? 1u << 16 : 0u) |
           (static_cast<uint32_t>(bn >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
}

// Nearest tf32 value (ties away from zero): add half a tf32 ulp to the
// magnitude bits and clear the 13 bits that tf32 drops.
__device__ __forceinline__ float tf32_rna(float v) {
    return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// Split 4 fp32 values into tf32 hi/lo parts and store them (16 bytes each) at
// byte `off` of the hi and lo tiles.
__device__ __forceinline__ void st_split4(char* tile_hi, char* tile_lo, uint32_t off,
                                          const float* v) {
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

// One K-block: the operand tiles of 8 reduction elements in shared memory (the
// B tiles only when A is in tensor memory).
template <int VM, int BN>
constexpr int b_off() {
    return Roles<BN>::TA ? 0 : TcTiles<VM>::na * 128 * 32;
}
template <int VM, int BN>
constexpr int block_bytes() {
    return b_off<VM, BN>() + TcTiles<VM>::nb * (BN / 2) * 32;
}
// Tensor-memory columns of one K-block's A tiles (8 per tile, TA only).
template <int VM>
constexpr int a_cols() {
    return TcTiles<VM>::na * 8;
}

// A stage holds kBlocks consecutive K-blocks (one per producer group); the MMA
// thread waits, issues and commits once per stage.
constexpr int kBlocks = 2;
template <int VM, int BN>
constexpr int stage_bytes() {
    return kBlocks * block_bytes<VM, BN>();
}

template <int VM, int BN>
constexpr int op_stages() {
    constexpr int by_smem = kStageBudget / stage_bytes<VM, BN>();
    constexpr int by_tmem = Roles<BN>::TA ? (512 - Roles<BN>::ACC_COLS) / (kBlocks * a_cols<VM>())
                                          : kMaxStages;
    constexpr int n = by_smem < by_tmem ? by_smem : by_tmem;
    return n < kMaxStages ? n : kMaxStages;
}

constexpr int kBarrierBytes = 512;
// The epilogue's per-warp transpose buffers (8 warps x 2 x 32 x 17 floats)
// reuse the operand stage area, which is at least this large.
constexpr int kEpiBytes = 8 * 2 * 32 * 17 * 4;

template <int VM, int BN>
constexpr int stage_area() {
    return op_stages<VM, BN>() * stage_bytes<VM, BN>() > kEpiBytes
               ? op_stages<VM, BN>() * stage_bytes<VM, BN>()
               : kEpiBytes;
}

// Weight sums of narrow tiles (LSQ, A in tensor memory) can take their raw
// operands from tensor-map bulk copies (TMA): per producer group a ring of
// kRawSlots K-blocks, each the A block (128 rows x 8 reduction elements) and
// the two B blocks (NC rows x 8) as fp32, followed by the ring's barriers.
constexpr int kRawSlots = 8;
template <int VM, int BN>
constexpr bool tma_capable() {
    return VM == LSQ && Roles<BN>::TA;
}
template <int BN>
constexpr int raw_slot_bytes() {
    return 128 * 32 + 2 * (BN / 2) * 32;
}
template <int VM, int BN>
constexpr int raw_area() {
    return tma_capable<VM, BN>() ? 2 * kRawSlots * raw_slot_bytes<BN>() + 2 * 2 * kRawSlots * 8 : 0;
}

template <int VM, int BN>
constexpr int smem_bytes() {
    return stage_area<VM, BN>() + kBarrierBytes + raw_area<VM, BN>();
}

// Tensor maps of the raw-operand copies (host-encoded; `on` = 0: the producers
// read global memory themselves). a: the A rows, 2-D (reduction innermost, row
// stride given); b0, b1: the two B operands of an NCHW delta tensor, 3-D
// (pixels of one image innermost, channels, images); L: pixels per image.
struct TmaArgs {
    CUtensorMap a, b0, b1;
    int on, L;
};

// Issue the MMAs of accumulator Q of one K-block: A tiles at descriptor da
// (shared memory) or, for TA tiles, at tensor-memory column da; B tiles at
// descriptor db.
template <int VM, int BN, int Q>
__device__ __forceinline__ void issue_acc(uint32_t d_tmem, uint64_t da, uint64_t db,
                                          uint32_t idesc, uint32_t accumulate) {
    using P = TcPlan<VM>;
    constexpr int A_TILE = 128 * 32, B_TILE = (BN / 2) * 32;
    constexpr int B0 = b_off<VM, BN>();
    bool first = true;
#pragma unroll
    for (int i = 0; i < P::n; ++i) {
        if (field(P::acc, i) != Q) continue;
        const uint64_t bd = db + static_cast<uint64_t>((B0 + field(P::b, i) * B_TILE) >> 4);
        if (Roles<BN>::TA) {
            mma_pair_tf32_ta(d_tmem, static_cast<uint32_t>(da) + field(P::a, i) * 8, bd, idesc,
                             first ? accumulate : 1u);
        } else {
            const uint64_t ad = da + static_cast<uint64_t>((field(P::a, i) * A_TILE) >> 4);
            mma_pair_tf32(d_tmem, ad, bd, idesc, first ? accumulate : 1u);
        }
        first = false;
    }
}

// 32 bytes at a 32-byte aligned address in one 256-bit load, not kept in L1.
// A warp of row-owning threads then reads whole 32-byte sectors; two 16-byte
// loads per row would touch each sector twice and slow the tensor pipe, whose
// operand reads share the SM's load/store path with these requests.
__device__ __forceinline__ void ld8(const float* p, float (&v)[8]) {
    asm volatile("ld.global.L1::no_allocate.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                   "=f"(v[6]), "=f"(v[7])
                 : "l"(p));
}

// The 8 floats at a 32-byte aligned p if `ok`, else zeros (one predicated
// 256-bit load, not kept in L1).
__device__ __forceinline__ void ld8_if(const float* p, bool ok, float (&v)[8]) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %9, 0;\n\t"
        "mov.b32 %0, 0;\n\tmov.b32 %1, 0;\n\tmov.b32 %2, 0;\n\tmov.b32 %3, 0;\n\t"
        "mov.b32 %4, 0;\n\tmov.b32 %5, 0;\n\tmov.b32 %6, 0;\n\tmov.b32 %7, 0;\n\t"
        "@q ld.global.L1::no_allocate.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t}"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
          "=f"(v[6]), "=f"(v[7])
        : "l"(p), "r"(static_cast<int>(ok)));
}

// *p if `ok`, else 0, as one predicated load into a zeroed register: the
// value is not consumed (no select waits on it) until the stage that uses it.
__device__ __forceinline__ float ldg_if(const float* p, bool ok) {
    float v;
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\tmov.b32 %0, 0;\n\t"
        "@q ld.global.cg.f32 %0, [%1];\n\t}"
        : "=f"(v)
        : "l"(p), "r"(static_cast<int>(ok)));
    return v;
}

// Staging of one operand side (A or B) of a stage: 2 operands x rows x 8
// reduction elements, spread over the side's threads of a producer group.
//   row mode (K-major tiles): a thread owns one tile row and loads its 8
//     elements, with one 256-bit load per operand when the row's elements are
//     contiguous and 32-byte aligned, else element by element;
//   chunk mode (MN-major tiles, 32-row multiples): when 4 consecutive rows are
//     contiguous and 16-byte aligned at every reduction index, a thread owns
//     chunks of (4 rows, 1 reduction index) and loads each with one 128-bit
//     load; 8 consecutive threads cover 32 rows at one index, 128 contiguous
//     bytes that also fill one 128-byte row of a tile atom.
// Element (row, k) of the side lies at base(row) + koff(k): A: arow.off(row) +
// k*ak; B: row*bn + brow.off(k).
struct Side {
    const float* p0;
    const float* p1;
    int row0, nrows;  // first global row of the CTA's tile part; rows of the matrix
    int ones_row;     // row of ones (A only; -1 if none)
    bool chunk;       // chunk mode (else row mode)
    bool vec;         // row mode: 256-bit loads
    bool gather;      // A: implicit patches of an NCHW image (row mode)
};

template <bool IS_A>
__device__ __forceinline__ int64_t row_base(const GemmArgs& g, int row) {
    return IS_A ? g.arow.off(row) : static_cast<int64_t>(row) * g.bn;
}
template <bool IS_A>
__device__ __forceinline__ int64_t k_off(const GemmArgs& g, int k) {
    return IS_A ? static_cast<int64_t>(k) * g.ak : g.brow.off(k);
}

// Element (row, k) of both operands (x and, if TWO, y); the bias row holds ones.
template <bool IS_A, bool TWO>
__device__ __forceinline__ void load_elem(const GemmArgs& g, const Side& sd, int row, int k,
                                          float& x, float& y) {
    x = 0.f;
    y = 0.f;
    if (row >= sd.nrows) return;
    if (IS_A && row == sd.ones_row) {
        x = 1.f;
        return;
    }
    const int64_t o = row_base<IS_A>(g, row) + k_off<IS_A>(g, k);
    x = __ldcg(sd.p0 + o);
    if (TWO) y = __ldcg(sd.p1 + o);
}

// Row mode: the 8 elements k0..k0+7 of `row`; zeros past kend. The reduction
// offsets of B go through brow with a single division per stage.
template <bool IS_A, bool TWO, int GM>
__device__ __forceinline__ void load_row(const GemmArgs& g, const Side& sd, int row,
                                         int64_t base, const GatherRow& gr, int k0, int kend,
                                         float (&v)[2][8]) {
    if (IS_A && sd.gather) {
        // implicit patches, reduction order (tap, c): one division per stage, then
        // addresses a channel plane apart and a bounds test per tap
        const Gather& ga = g.ga;
        const int64_t plane = static_cast<int64_t>(ga.H) * ga.W;
        int tap = k0 / ga.C, c = k0 - tap * ga.C;
        int kh = tap / ga.k, kw = tap - kh * ga.k;
        int ih, iw;
        bool inside = row < sd.nrows && gather_tap<GM>(ga, gr, kh, kw, &ih, &iw);
        if (ga.nhwc) {
            // channels-last: the block's 8 channels of one tap are contiguous
            int64_t o = gr.base + (static_cast<int64_t>(ih) * ga.W + iw) * ga.C + c;
            if (ga.C % 8 == 0 && k0 + 8 <= kend) {
                ld8_if(sd.p0 + o, inside, v[0]);
                if (TWO) {
                    ld8_if(sd.p1 + o, inside, v[1]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[1][j] = 0.f;
                }
                return;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool ok = inside && k0 + j < kend;
                v[0][j] = ldg_if(sd.p0 + o, ok);
                v[1][j] = TWO ? ldg_if(sd.p1 + o, ok) : 0.f;
                ++o;
                if (++c == ga.C) {
                    c = 0;
                    if (++kw == ga.k) {
                        kw = 0;
                        ++kh;
                    }
                    inside = row < sd.nrows && gather_tap<GM>(ga, gr, kh, kw, &ih, &iw);
                    o = gr.base + (static_cast<int64_t>(ih) * ga.W + iw) * ga.C;
                }
            }
            return;
        }
        int64_t o = gr.base + (static_cast<int64_t>(c) * ga.H + ih) * ga.W + iw;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const bool ok = inside && k0 + j < kend;
            v[0][j] = ldg_if(sd.p0 + o, ok);
            v[1][j] = TWO ? ldg_if(sd.p1 + o, ok) : 0.f;
            o += plane;
            if (++c == ga.C) {
                c = 0;
                if (++kw == ga.k) {
                    kw = 0;
                    ++kh;
                }
                inside = row < sd.nrows && gather_tap<GM>(ga, gr, kh, kw, &ih, &iw);
                o = gr.base + static_cast<int64_t>(ih) * ga.W + iw;
            }
        }
        return;
    }
    const bool one = IS_A && row == sd.ones_row;
    if (sd.vec && k0 + 8 <= kend && row < sd.nrows && !one) {
        const int64_t o = base + k_off<IS_A>(g, k0);
        ld8(sd.p0 + o, v[0]);
        if (TWO) ld8(sd.p1 + o, v[1]);
        return;
    }
    const RowMap& m = g.brow;
    uint32_t q = 0, r = 0;
    if (!IS_A && m.div > 0) {
        q = static_cast<uint32_t>(k0) / static_cast<uint32_t>(m.div);
        r = static_cast<uint32_t>(k0) - q * static_cast<uint32_t>(m.div);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int k = k0 + j;
        const bool in = k < kend && row < sd.nrows;
        const int64_t ko =
            IS_A ? static_cast<int64_t>(k) * g.ak
                 : (m.div > 0 ? static_cast<int64_t>(q) * m.outer + static_cast<int64_t>(r) * m.stride
                              : static_cast<int64_t>(k) * m.stride);
        v[0][j] = one ? (in ? 1.f : 0.f) : ldg_if(sd.p0 + base + ko, in);
        v[1][j] = (TWO && !one) ? ldg_if(sd.p1 + base + ko, in) : 0.f;
        if (!IS_A && m.div > 0 && ++r == static_cast<uint32_t>(m.div)) {
            r = 0;
            ++q;
        }
    }
}

// Chunk mode: rows r..r+3 at reduction index k into v[o][4*slot .. 4*slot+3].
template <bool IS_A, bool TWO>
__device__ __forceinline__ void load_chunk(const GemmArgs& g, const Side& sd, int r, int k,
                                           int kend, int slot, float (&v)[2][8]) {
    float* x = &v[0][4 * slot];
    float* y = &v[1][4 * slot];
    if (k >= kend) {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = y[e] = 0.f;
        return;
    }
    const bool whole = r + 3 < sd.nrows && !(IS_A && sd.ones_row >= r && sd.ones_row <= r + 3);
    if (whole) {
        const int64_t o = row_base<IS_A>(g, r) + k_off<IS_A>(g, k);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(sd.p0 + o));
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        if (TWO) {
            const float4 b = __ldcg(reinterpret_cast<const float4*>(sd.p1 + o));
            y[0] = b.x; y[1] = b.y; y[2] = b.z; y[3] = b.w;
        }
        return;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) load_elem<IS_A, TWO>(g, sd, r + e, k, x[e], y[e]);
}

// Forms the operand tiles of one side from 4 values per operand (x, y) and
// stores them at byte `off` of each tile (tile t at st + t * tile_bytes).
template <int VM, bool IS_A>
__device__ __forceinline__ void store_tiles(char* st, int tile_bytes, uint32_t off, const float* x,
                                            const float* y) {
    float sq[4];
    char* t0 = st;
    st_split4(t0, t0 + tile_bytes, off, x);
    if (IS_A) {
        if (VM == FULL || VM == LSQ) {
#pragma unroll
            for (int e = 0; e < 4; ++e) sq[e] = x[e] * x[e];
            st_split4(t0 + 2 * tile_bytes, t0 + 3 * tile_bytes, off, sq);
        }
        if (VM == FULL) st_split4(t0 + 4 * tile_bytes, t0 + 5 * tile_bytes, off, y);
        if (VM == RSQ) st_split4(t0 + 2 * tile_bytes, t0 + 3 * tile_bytes, off, y);
    } else {
        if (VM == FULL) {
            st_split4(t0 + 2 * tile_bytes, t0 + 3 * tile_bytes, off, y);
#pragma unroll
            for (int e = 0; e < 4; ++e) sq[e] = x[e] * x[e] + y[e];
            st_split4(t0 + 4 * tile_bytes, t0 + 5 * tile_bytes, off, sq);
        } else if (VM == RSQ) {
#pragma unroll
            for (int e = 0; e < 4; ++e) sq[e] = x[e] * x[e];
            st_split4(t0 + 2 * tile_bytes, t0 + 3 * tile_bytes, off, sq);
        } else {
            st_split4(t0 + 2 * tile_bytes, t0 + 3 * tile_bytes, off, y);
        }
    }
}

// Chunk mode is possible when 4 consecutive rows are adjacent and 16-byte
// aligned for every reduction index.
template <bool IS_A>
__device__ __forceinline__ bool chunk_ok(const GemmArgs& g, const float* p0, const float* p1) {
    const uintptr_t al = (reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1)) & 15;
    if (al) return false;
    if (IS_A) {
        const RowMap& m = g.arow;
        return m.stride == 1 && g.ak % 4 == 0 && (m.div <= 0 || (m.div % 4 == 0 && m.outer % 4 == 0));
    }
    const RowMap& m = g.brow;
    return g.bn == 1 && m.stride % 4 == 0 && (m.div <= 0 || m.outer % 4 == 0);
}

// Row mode with 256-bit loads is possible when each row's reduction elements
// are contiguous and every 8-element run starts 32-byte aligned.
template <bool IS_A>
__device__ __forceinline__ bool rowvec_ok(const GemmArgs& g, const float* p0, const float* p1) {
    const uintptr_t al = (reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1)) & 31;
    if (al) return false;
    if (IS_A) {
        const RowMap& m = g.arow;
        return g.ak == 1 && m.stride % 8 == 0 && (m.div <= 0 || m.outer % 8 == 0);
    }
    const RowMap& m = g.brow;
    return m.stride == 1 && g.bn % 8 == 0 && (m.div <= 0 || (m.div % 8 == 0 && m.outer % 8 == 0));
}

// Number of chunks and last stage of chunk c when chunk boundaries are shifted
// by `o` stages (chunk c covers stages [c*kChunk - o, (c+1)*kChunk - o)).
__device__ __forceinline__ int num_chunks(int niter, int o) { return (niter + o + kChunk - 1) / kChunk; }
__device__ __forceinline__ int chunk_end(int c, int o, int niter) {
    return min((c + 1) * kChunk - o, niter) - 1;
}

struct ProdCtx {
    char* smem;
    uint64_t* empty;
    uint64_t* bfull;  // prepared-B copies of each stage slot (local)
    uint32_t full0;  // cluster address of the leader CTA's full barriers
    Abort ab;
    int niter, kbeg, kend;
    int grp;  // producer group: stages of parity grp
    int t;    // thread index within the group's threads of this side
    int lane;
    uint32_t tmem;  // tensor-memory base (A stages of TA tiles)
    // raw operands by tensor-map copies (tm != nullptr): this group's ring of
    // kRawSlots K-blocks and its barriers; `issuer` = the thread that issues the
    // copies; a_row0 / b_row0: the CTA's first A row and B row (column)
    const TmaArgs* tm;
    char* raw;
    uint64_t* rfull;
    uint64_t* rempty;
    bool issuer;
    int a_row0, b_row0;
};

// Tensor-map copies of the raw operands of K-block `it` into ring slot `slot`:
// the A block (128 rows) and both B blocks (NC rows of one image's pixels).
template <int BN>
__device__ __forceinline__ void tma_issue(const ProdCtx& c, int it, int slot) {
    constexpr int NC = BN / 2;
    const uint32_t base = smem_u32(c.raw + slot * raw_slot_bytes<BN>());
    uint64_t* bar = &c.rfull[slot];
    mbar_expect_tx(bar, static_cast<uint32_t>(raw_slot_bytes<BN>()));
    const int k0 = c.kbeg + it * kBK;
    tma_load_2d(base, &c.tm->a, k0, c.a_row0, bar);
    const int img = k0 / c.tm->L, px = k0 - img * c.tm->L;
    tma_load_3d(base + 128 * 32, &c.tm->b0, px, c.b_row0, img, bar);
    tma_load_3d(base + 128 * 32 + NC * 32, &c.tm->b1, px, c.b_row0, img, bar);
}

// One side's producer thread: K-blocks grp, grp+2, ... with prefetch_depth of them loaded
// ahead into registers.
template <int VM, int BN, bool IS_A, int GM>
__device__ __forceinline__ void producer(const GemmArgs& g, const ProdCtx& c, const Side& sd) {
    using R = Roles<BN>;
    constexpr int ROWS = IS_A ? 128 : R::NC;
    constexpr int NTH = IS_A ? 128 : 32 * R::BW;  // this side's threads in a group
    constexpr int GROUPS = ROWS / 4;               // chunk mode: 4-row groups
    constexpr int SLOTS = GROUPS * 8;              // (4 rows, 1 k) chunks of a stage
    constexpr int SPT = (SLOTS + NTH - 1) / NTH;   // chunks per thread
    static_assert(SPT >= 1 && SPT <= 2, "chunk slots per thread");
    constexpr int TILE = ROWS * 32;
    constexpr int STAGE = stage_bytes<VM, BN>();
    constexpr int BLOCK = block_bytes<VM, BN>();
    constexpr int OPS = op_stages<VM, BN>();
    constexpr int OFF = IS_A ? 0 : b_off<VM, BN>();  // the side's first tile
    constexpr bool TMEM_A = IS_A && R::TA;          // A rows go to tensor memory
    constexpr bool TWO = IS_A ? VM != LSQ : VM != RSQ;
    const bool has_row = c.t < ROWS;
    const int row = sd.row0 + c.t;
    const bool row_in = has_row && row < sd.nrows;
    const int64_t base =
        (row_in && !(IS_A && (row == sd.ones_row || sd.gather))) ? row_base<IS_A>(g, row) : 0;
    GatherRow gr{0, 0, 0};
    if (IS_A && sd.gather) gr = gather_row(g.ga, row_in ? row : 0);

    auto load = [&](int it, float (&v)[2][8]) {
        if (it >= c.niter) return;
        const int k0 = c.kbeg + it * kBK;
        if (sd.chunk) {
#pragma unroll
            for (int j = 0; j < SPT; ++j) {
                const int slot = c.t + j * NTH;
                if (slot < SLOTS)
                    load_chunk<IS_A, TWO>(g, sd, sd.row0 + (slot % GROUPS) * 4, k0 + slot / GROUPS,
                                          c.kend, j, v);
            }
        } else if (has_row) {
            load_row<IS_A, TWO, GM>(g, sd, row, base, gr, k0, c.kend, v);
        }
    };
    // K-block `it` is block it % kBlocks of stage it / kBlocks (= this group's
    // half of that stage's slot).
    auto produce = [&](int it, const float (&v)[2][8]) -> bool {
        const int S = it / kBlocks, s = S % OPS;
        if (S >= OPS && !warp_wait(&c.empty[s], ((S / OPS) - 1) & 1, c.ab, 1)) return false;
        // Rows outside the matrix are not written: an output row (column)
        // depends only on its own A row (B row), and those outputs are dropped.
        if (TMEM_A) {
            // this thread's row is its lane of the warp's tensor-memory quarter
            // (warp % 4 == row / 32); the tiles' 8 reduction elements are 8
            // consecutive columns
            tc_fence_after();  // after the MMAs that read this slot (empty barrier)
            // tcgen05.st is warp-collective: every lane stores; rows past M hold
            // zeros (load_row) and their outputs are dropped
            const uint32_t col = R::A0 + static_cast<uint32_t>(
                                             (s * kBlocks + it % kBlocks) * a_cols<VM>());
            const uint32_t ta = c.tmem + (static_cast<uint32_t>(c.t & ~31) << 16) + col;
            float sq[8];
            // a tile's hi and lo parts are 16 consecutive columns: one 16-column store
            auto put = [&](int t, const float (&x)[8]) {
                float hl[16];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    hl[e] = tf32_rna(x[e]);
                    hl[8 + e] = tf32_rna(x[e] - hl[e]);
                }
                tmem_st16(ta + t * 16, hl);
            };
            put(0, v[0]);
            if (VM == FULL || VM == LSQ) {
#pragma unroll
                for (int e = 0; e < 8; ++e) sq[e] = v[0][e] * v[0][e];
                put(1, sq);
            }
            if (VM == FULL) put(2, v[1]);
            if (VM == RSQ) put(1, v[1]);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (c.lane == 0) arrive_cluster(c.full0 + static_cast<uint32_t>(s * 8));
            return true;
        }
        char* st = c.smem + s * STAGE + (it % kBlocks) * BLOCK + OFF;
        bool wrote = false;
        if (sd.chunk) {
#pragma unroll
            for (int j = 0; j < SPT; ++j) {
                const int slot = c.t + j * NTH;
                const int r = (slot % GROUPS) * 4;
                if (slot < SLOTS && sd.row0 + r < sd.nrows) {
                    store_tiles<VM, IS_A>(st, TILE, tile_off_mn(r, slot / GROUPS, ROWS),
                                          &v[0][4 * j], &v[1][4 * j]);
                    wrote = true;
                }
            }
        } else if (row_in) {
            store_tiles<VM, IS_A>(st, TILE, tile_off_k(c.t, 0), &v[0][0], &v[1][0]);
            store_tiles<VM, IS_A>(st, TILE, tile_off_k(c.t, 4), &v[0][4], &v[1][4]);
            wrote = true;
        }
        if (wrote) fence_proxy_async();
        __syncwarp();
        if (c.lane == 0) arrive_cluster(c.full0 + static_cast<uint32_t>(s * 8));
        return true;
    };

    bool alive = true;
    if (tma_capable<VM, BN>() && c.tm != nullptr) {
        // Raw operands arrive by tensor-map copies kRawSlots K-blocks ahead; each
        // thread reads its row's 8 elements from the ring slot, the group's warps
        // release the slot, and the issuer refills it with the group's K-block
        // kRawSlots later.
        const int nj = c.niter > c.grp ? (c.niter - c.grp + 1) / 2 : 0;
        int issued = 0;
        if (c.issuer) {
            for (; issued < nj && issued < kRawSlots; ++issued)
                if (c.lane == 0) tma_issue<BN>(c, c.grp + 2 * issued, issued);
            __syncwarp();
        }
        for (int j = 0; j < nj && alive; ++j) {
            const int it = c.grp + 2 * j;
            if (c.issuer && j >= 1 && issued < nj) {
                // slot of K-block j - 1: free once every warp of the group read it
                const int pj = j - 1, ps = pj % kRawSlots;
                if (!warp_wait(&c.rempty[ps], (pj / kRawSlots) & 1, c.ab, 7)) break;
                if (c.lane == 0) tma_issue<BN>(c, c.grp + 2 * issued, issued % kRawSlots);
                __syncwarp();
                ++issued;
            }
            const int sl = j % kRawSlots;
            if (!warp_wait(&c.rfull[sl], (j / kRawSlots) & 1, c.ab, 8)) break;
            float v[2][8];
            const float* src = reinterpret_cast<const float*>(c.raw + sl * raw_slot_bytes<BN>()) +
                               (IS_A ? 0 : 128 * 8);
            const int k0 = c.kbeg + it * kBK;
            if (has_row) {
                const float4* p0 = reinterpret_cast<const float4*>(src + c.t * 8);
                const float4 a0 = p0[0], a1 = p0[1];
                const float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                float y[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (!IS_A) {
                    const float4* p1 = reinterpret_cast<const float4*>(src + ROWS * 8 + c.t * 8);
                    const float4 b0 = p1[0], b1 = p1[1];
                    y[0] = b0.x; y[1] = b0.y; y[2] = b0.z; y[3] = b0.w;
                    y[4] = b1.x; y[5] = b1.y; y[6] = b1.z; y[7] = b1.w;
                }
                const bool one = IS_A && row == sd.ones_row;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const bool in = k0 + e < c.kend;  // past the split's end: zero
                    v[0][e] = in ? (one ? 1.f : x[e]) : 0.f;
                    v[1][e] = in ? y[e] : 0.f;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[0][e] = v[1][e] = 0.f;
            }
            __syncwarp();
            if (c.lane == 0) mbar_arrive_local(&c.rempty[sl]);
            alive = produce(it, v);
        }
        // copies issued but not consumed (after an abort) land before the CTA exits
        if (c.issuer) {
            const int first = issued > kRawSlots ? issued - kRawSlots : 0;
            for (int j = first; j < issued; ++j)
                mbar_drain(&c.rfull[j % kRawSlots], (j / kRawSlots) & 1);
        }
    }
    constexpr int kDepth = prefetch_depth<BN>();
    float buf[kDepth][2][8];
    if (!(tma_capable<VM, BN>() && c.tm != nullptr)) {
#pragma unroll
        for (int d = 0; d < kDepth; ++d) load(c.grp + 2 * d, buf[d]);
    }
    for (int it0 = c.grp; it0 < c.niter && alive && !(tma_capable<VM, BN>() && c.tm != nullptr);
         it0 += 2 * kDepth) {
#pragma unroll
        for (int d = 0; d < kDepth; ++d) {
            const int it = it0 + 2 * d;
            if (it < c.niter && alive) {
                alive = produce(it, buf[d]);
                load(it + 2 * kDepth, buf[d]);
            }
        }
    }
    // An odd number of K-blocks leaves the last stage's second block empty; its
    // group still arrives so that the stage completes.
    if (alive && c.grp == 1 && (c.niter & 1)) {
        const int S = c.niter / kBlocks, s = S % OPS;
        if (S < OPS || warp_wait(&c.empty[s], ((S / OPS) - 1) & 1, c.ab, 1)) {
            __syncwarp();
            if (c.lane == 0) arrive_cluster(c.full0 + static_cast<uint32_t>(s * 8));
        }
    }
}

// B side from prepared tiles (g.bpk), two warps per CTA:
//   issuer (role 0): as each stage slot frees, copies the stage's K-blocks of B
//     tiles of this CTA's NC columns (contiguous, in shared-memory byte order),
//     one bulk copy per K-block, completing on the slot's bfull barrier;
//   forwarder (role 1): as each stage's copies land, arrives on the leader's full
//     barrier of the stage for the whole B side of this CTA.
// Neither waits for the other, so copies run as far ahead as the free slots
// allow and a landed stage is forwarded at once.
template <int VM, int BN>
__device__ __forceinline__ void packed_b(const GemmArgs& g, const ProdCtx& c, int chunk,
                                         int role) {
    using R = Roles<BN>;
    constexpr uint32_t KB_BYTES = TcTiles<VM>::nb * R::NC * 32;
    constexpr int STAGE = stage_bytes<VM, BN>();
    constexpr int BLOCK = block_bytes<VM, BN>();
    constexpr int OPS = op_stages<VM, BN>();
    constexpr int OFF = b_off<VM, BN>();
    const int nst = (c.niter + kBlocks - 1) / kBlocks;
    if (role == 1) {
        for (int F = 0; F < nst; ++F) {
            const int f = F % OPS;
            if (!warp_wait(&c.bfull[f], (F / OPS) & 1, c.ab, 6)) return;
            __syncwarp();
            if (c.lane == 0) arrive_cluster(c.full0 + static_cast<uint32_t>(f * 8));
        }
        return;
    }
    const char* src0 =
        g.bpk + (static_cast<int64_t>(chunk) * g.bpk_nkb + c.kbeg / kBK) * KB_BYTES;
    int issued = 0;
    for (int S = 0; S < nst; ++S) {
        const int s = S % OPS;
        if (S >= OPS && !warp_wait(&c.empty[s], ((S / OPS) - 1) & 1, c.ab, 1)) break;
        if (c.lane == 0) {
            const int nblk = min(kBlocks, c.niter - S * kBlocks);
            mbar_expect_tx(&c.bfull[s], nblk * KB_BYTES);
            const uint32_t dst = smem_u32(c.smem + s * STAGE + OFF);
            for (int sub = 0; sub < nblk; ++sub)
                bulk_g2s(dst + sub * BLOCK, src0 + static_cast<int64_t>(S * kBlocks + sub) * KB_BYTES,
                         KB_BYTES, &c.bfull[s]);
        }
        __syncwarp();
        issued = S + 1;
    }
    // The copies of the last stages issued (the latest phase of each slot) must
    // land before the CTA may exit, also after an abort.
    for (int F = max(0, issued - OPS); F < issued; ++F)
        mbar_drain(&c.bfull[F % OPS], (F / OPS) & 1);
}

// GM: the A gather compiled in (0 patches, 1 col2im of any stride, 2 col2im of
// stride 1); operands that are not gathered ignore it.
template <int VM, bool MEAN, int EPI, int BN, int GM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Roles<BN>::THREADS, 1)
    moment_tc_kernel(const GemmArgs g, const __grid_constant__ TmaArgs tm) {
    using R = Roles<BN>;
    using T = TcTiles<VM>;
    constexpr int A_TILE = 128 * 32, B_TILE = R::NC * 32;
    constexpr int STAGE = stage_bytes<VM, BN>();
    constexpr int BLOCK = block_bytes<VM, BN>();
    constexpr int OPS = op_stages<VM, BN>();
    constexpr int NP = R::NP;
    constexpr int kOff1 = kChunk / 2;  // stage shift of the variance chunks
    extern __shared__ __align__(1024) char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + stage_area<VM, BN>());  // [OPS], leader only
    uint64_t* empty = full + kMaxStages;                                // [OPS]
    uint64_t* chunk_full = empty + kMaxStages;                          // [q*2 + b]
    uint64_t* chunk_empty = chunk_full + 4;                             // [q*2 + b], leader
    uint64_t* done = chunk_empty + 4;
    uint64_t* bfull = done + 1;  // [OPS], prepared-B copies
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bfull + kMaxStages);
    volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // raw-operand rings (tensor-map copies), one per producer group
    constexpr bool kTma = tma_capable<VM, BN>();
    char* raw = smem + stage_area<VM, BN>() + kBarrierBytes;
    uint64_t* rfull = reinterpret_cast<uint64_t*>(raw + 2 * kRawSlots * raw_slot_bytes<BN>());
    uint64_t* rempty = rfull + 2 * kRawSlots;  // [grp * kRawSlots + slot]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int m_cta = static_cast<int>(blockIdx.x >> 1) * 256 + static_cast<int>(rank) * 128;
    const int n0 = blockIdx.y * BN;
    const int batch = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
    const int kbeg = split * g.kchunk;
    const int kend = min(g.Kr, kbeg + g.kchunk);
    const int niter = kend > kbeg ? (kend - kbeg + kBK - 1) / kBK : 0;
    const Abort ab{abort_word, map_to(smem_u32(const_cast<int*>(abort_word)), rank ^ 1u)};
    // Prepared B tiles (FULL and RSQ, unbatched): one arrival per CTA for the B side.
    const bool packed = g.bpk != nullptr && g.bpk_nc == R::NC;
    const bool use_tma = kTma && tm.on != 0 && !packed;

    if (tid == 0) {
        for (int s = 0; s < OPS; ++s) {
            mbar_init(&full[s], packed ? 2 * 2 * 4 + 2 : R::STAGE_ARRIVALS);
            mbar_init(&empty[s], 1);
            mbar_init(&bfull[s], 1);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(&chunk_full[i], 1);
            mbar_init(&chunk_empty[i], 16);  // 8 accumulator warps in each CTA
        }
        mbar_init(done, 1);
        if (use_tma) {
            for (int i = 0; i < 2 * kRawSlots; ++i) {
                mbar_init(&rfull[i], 1);
                mbar_init(&rempty[i], 4 + R::BW);  // the group's A and B producer warps
            }
        }
        *abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == R::MMA_W) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(R::COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();  // barriers initialised and tensor memory allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // operand sides of this CTA (uniform over the CTA)
    constexpr bool TWO_A = VM != LSQ, TWO_B = VM != RSQ;
    Side sa, sb;
    sa.p0 = g.x + batch * g.a_bs;
    sa.p1 = TWO_A ? g.y + batch * g.a_bs : sa.p0;
    sa.row0 = m_cta;
    sa.nrows = g.M;
    sa.ones_row = g.ones_row;
    sa.gather = g.ga.on != 0;
    sa.vec = !sa.gather && rowvec_ok<true>(g, sa.p0, sa.p1);
    // tensor-memory A rows are owned by one thread each: row mode
    sa.chunk = !R::TA && !sa.gather && !sa.vec && chunk_ok<true>(g, sa.p0, sa.p1);
    sb.p0 = g.u + batch * g.b_bs;
    sb.p1 = TWO_B ? g.v + batch * g.b_bs : sb.p0;
    sb.row0 = n0 + static_cast<int>(rank) * R::NC;
    sb.nrows = g.N;
    sb.ones_row = -1;
    sb.gather = false;
    sb.vec = rowvec_ok<false>(g, sb.p0, sb.p1);
    sb.chunk = R::NC % 32 == 0 && !sb.vec && chunk_ok<false>(g, sb.p0, sb.p1);

    if (warp < R::MMA_W) {
        // ------------------------------------------------------------ producers
        const bool is_a = warp < R::B_W0;
        ProdCtx c;
        c.smem = smem;
        c.empty = empty;
        c.full0 = map_to(smem_u32(full), 0);  // the leader's full barriers
        c.ab = ab;
        c.niter = niter;
        c.kbeg = kbeg;
        c.kend = kend;
        c.lane = lane;
        c.tmem = tmem;
        c.tm = nullptr;
        if (use_tma) {
            const int grp = is_a ? (warp >> 2) : (warp - R::B_W0) / R::BW;
            c.tm = &tm;
            c.raw = raw + grp * kRawSlots * raw_slot_bytes<BN>();
            c.rfull = rfull + grp * kRawSlots;
            c.rempty = rempty + grp * kRawSlots;
            c.issuer = is_a && (warp & 3) == 0;
            c.a_row0 = sa.row0;
            c.b_row0 = sb.row0;
        }
        if (is_a) {
            c.grp = warp >> 2;
            c.t = (warp & 3) * 32 + lane;
            producer<VM, BN, true, GM>(g, c, sa);
        } else if (packed) {
            c.bfull = bfull;
            if (warp < R::B_W0 + 2) packed_b<VM, BN>(g, c, sb.row0 / R::NC, warp - R::B_W0);
        } else {
            c.grp = (warp - R::B_W0) / R::BW;
            c.t = ((warp - R::B_W0) % R::BW) * 32 + lane;
            producer<VM, BN, false, GM>(g, c, sb);
        }
    } else if (warp == R::MMA_W) {
        // ------------------------------------------------------------ MMA issue
        // The whole warp runs the loop (its state stays warp-uniform, so the
        // descriptors live in uniform registers) and one elected lane issues the
        // single-thread tcgen05.mma / tcgen05.commit instructions. Run by one lane
        // alone, the same loop fed the tensor pipe at half its rate.
        if (leader) {
            const bool el = elect_one();
            // A of TA tiles: tensor-memory column of the stage's first tile
            const uint64_t da_first =
                R::TA ? static_cast<uint64_t>(tmem + R::A0) : smem_desc(smem_u32(smem), sa.chunk, 128);
            constexpr uint64_t kDaBlock = R::TA ? a_cols<VM>() : (BLOCK >> 4);
            constexpr uint64_t kDaStage = R::TA ? kBlocks * a_cols<VM>() : (STAGE >> 4);
            // prepared tiles: MN-major (swizzled) when NC allows it, else K-major
            const bool b_mn = packed ? R::NC % 32 == 0 : sb.chunk;
            const uint64_t db_first = smem_desc(smem_u32(smem), b_mn, R::NC);
            const uint32_t idesc = instr_desc(BN, sa.chunk, b_mn);
            uint64_t da = da_first, db = db_first;
            int s = 0;
            uint32_t ph = 0;
            int nit = niter;
            if (*const_cast<volatile int*>(&g_force_abort)) {
                // test hook: give up the tiles as a wait that ran out would
                if (el) {
                    *ab.flag = 1;
                    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(ab.peer), "r"(1) : "memory");
                    atomicCAS(&g_device_error, 0, 2);
                }
                __syncwarp();
                nit = 0;
            }
            int pos0 = 0, pos1 = kOff1;  // (stage + shift) % kChunk of each accumulator
            int c0 = 0, c1 = 0;          // chunk index of each accumulator
            // An accumulator whose chunk buffer must first be drained by a fold
            // goes second, so that the other one's products keep the pipe busy.
            auto drained = [&](int q, int c) -> bool {
                if (!warp_wait(&chunk_empty[q * 2 + c % NP], ((c / NP) - 1) & 1, ab, 5)) return false;
                tc_fence_after();
                return true;
            };
            for (int it0 = 0; it0 < nit; it0 += kBlocks) {
                if (!warp_wait(&full[s], ph, ab, 2)) break;
                tc_fence_after();
                bool ok = true;
#pragma unroll
                for (int sub = 0; sub < kBlocks; ++sub) {
                    const int it = it0 + sub;
                    if (it >= niter || !ok) break;
                    const uint64_t bda = da + sub * kDaBlock;
                    const uint64_t bdb = db + static_cast<uint64_t>((sub * BLOCK) >> 4);
                    const bool first0 = pos0 == 0, first1 = it == 0 || pos1 == 0;
                    const bool last0 = it == niter - 1 || pos0 == kChunk - 1;
                    const bool last1 = it == niter - 1 || pos1 == kChunk - 1;
                    const int b0 = c0 % NP, b1 = c1 % NP;
                    const uint32_t acc0 = first0 ? 0u : 1u, acc1 = first1 ? 0u : 1u;
                    if (!(MEAN && first0 && c0 >= NP)) {
                        if (MEAN && el) issue_acc<VM, BN, 0>(tmem + R::pcol(0, b0), bda, bdb, idesc, acc0);
                        if (first1 && c1 >= NP) ok = drained(1, c1);
                        if (ok && el) issue_acc<VM, BN, 1>(tmem + R::pcol(1, b1), bda, bdb, idesc, acc1);
                    } else {
                        if (el) issue_acc<VM, BN, 1>(tmem + R::pcol(1, b1), bda, bdb, idesc, acc1);
                        ok = drained(0, c0);
                        if (ok && el) issue_acc<VM, BN, 0>(tmem + R::pcol(0, b0), bda, bdb, idesc, acc0);
                    }
                    if (!ok) break;
                    if (MEAN && last0 && el) mma_commit_pair(&chunk_full[b0]);
                    if (last1 && el) mma_commit_pair(&chunk_full[2 + b1]);
                    if (++pos0 == kChunk) { pos0 = 0; ++c0; }
                    if (++pos1 == kChunk) { pos1 = 0; ++c1; }
                }
                if (!ok) break;
                if (el) mma_commit_pair(&empty[s]);
                __syncwarp();
                if (++s == OPS) {
                    s = 0;
                    ph ^= 1u;
                    da = da_first;
                    db = db_first;
                } else {
                    da += kDaStage;
                    db += static_cast<uint64_t>(STAGE >> 4);
                }
            }
            if (el) mma_commit_pair(done);  // arrives once every MMA issued above completed
            __syncwarp();
        }
    } else {
        // -------------------------------------------- accumulator warps
        const int a = warp - R::ACC_W0;
        const int sub = warp & 3;  // tensor-memory lane quarter this warp may access
        constexpr int HC = BN / 2;  // columns per warp per accumulator
        const int cbeg = (a >> 2) * HC;
        const int row = m_cta + sub * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(sub * 32) << 16);
        const uint32_t ce0 = map_to(smem_u32(chunk_empty), 0);  // the leader's drain barriers
        const int64_t ro = (EPI == EPI_STORE && row < g.M) ? g.orow.off(row) + batch * g.o_bs : 0;
        const int nch0 = num_chunks(niter, 0), nch1 = num_chunks(niter, kOff1);
        int c0 = MEAN ? 0 : nch0, c1 = 0;
        bool ok = niter > 0;
        while (ok) {
            const bool fin0 = !MEAN || c0 == nch0 - 1;
            const bool fin1 = c1 == nch1 - 1;
            if (fin0 && fin1) break;
            const int e0 = fin0 ? INT_MAX : chunk_end(c0, 0, niter);
            const int e1 = fin1 ? INT_MAX : chunk_end(c1, kOff1, niter);
            const int q = e0 <= e1 ? 0 : 1;
            const int cq = q ? c1 : c0, bq = cq % NP;
            // intermediate fold of chunk cq of accumulator q: T_q += P_q
            ok = warp_wait(&chunk_full[q * 2 + bq], (cq / NP) & 1, ab, 3);
            if (!ok) break;
            tc_fence_after();
            const uint32_t pc = lane_base + R::pcol(q, bq) + cbeg;
            const uint32_t tc = lane_base + R::tcol(q) + cbeg;
#pragma unroll 1
            for (int k = 0; k < HC; k += 16) {
                uint32_t pr[16], tr[16];
                tmem_ld16(pc + k, pr);
                if (cq > 0) tmem_ld16(tc + k, tr);
                tmem_wait_ld();
                if (k + 16 >= HC) {
                    // this warp has read all of its part of the chunk buffer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) arrive_cluster(ce0 + static_cast<uint32_t>((q * 2 + bq) * 8));
                }
                float tv[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    tv[j] = cq > 0 ? __uint_as_float(tr[j]) + __uint_as_float(pr[j])
                                   : __uint_as_float(pr[j]);
                tmem_st16(tc + k, tv);
            }
            tmem_wait_st();
            if (q) ++c1;
            else ++c0;
        }
        if (ok) {
            // last chunks of both accumulators: fold and run the epilogue
            const int b0 = (MEAN ? c0 : 0) % NP, b1 = c1 % NP;
            if (MEAN) ok = warp_wait(&chunk_full[b0], (c0 / NP) & 1, ab, 3);
            if (ok) ok = warp_wait(&chunk_full[2 + b1], (c1 / NP) & 1, ab, 3);
            if (ok) {
                tc_fence_after();
                // Outputs whose columns are contiguous (row-major stores, split
                // partials, weight parameters) go through a per-warp transpose in
                // shared memory (the operand stages are idle once the last MMAs
                // completed), so that a warp touches 2 rows x 16 consecutive columns
                // per access instead of 32 rows x 1 column. Outputs contiguous
                // along the rows (NCHW) keep the row-per-lane order.
                const bool transpose = EPI != EPI_STORE || g.on == 1;
                float* eb = reinterpret_cast<float*>(smem) + a * (2 * 32 * 17);
#pragma unroll 1
                for (int k = 0; k < HC; k += 16) {
                    uint32_t pm[16], pv[16], tm[16], tv[16];
                    if (MEAN) tmem_ld16(lane_base + R::pcol(0, b0) + cbeg + k, pm);
                    tmem_ld16(lane_base + R::pcol(1, b1) + cbeg + k, pv);
                    if (MEAN && c0 > 0) tmem_ld16(lane_base + R::tcol(0) + cbeg + k, tm);
                    if (c1 > 0) tmem_ld16(lane_base + R::tcol(1) + cbeg + k, tv);
                    tmem_wait_ld();
                    float vm[16], vv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        vm[j] = MEAN ? (c0 > 0 ? __uint_as_float(tm[j]) + __uint_as_float(pm[j])
                                               : __uint_as_float(pm[j]))
                                     : 0.f;
                        vv[j] = c1 > 0 ? __uint_as_float(tv[j]) + __uint_as_float(pv[j])
                                       : __uint_as_float(pv[j]);
                    }
                    if (transpose) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            eb[lane * 17 + j] = vm[j];
                            eb[32 * 17 + lane * 17 + j] = vv[j];
                        }
                        __syncwarp();
                        const int cl = lane & 15, col = n0 + cbeg + k + cl;
#pragma unroll 4
                        for (int i = 0; i < 16; ++i) {
                            const int rl = 2 * i + (lane >> 4);
                            const int r = m_cta + sub * 32 + rl;
                            if (r < g.M && col < g.N) {
                                const int64_t rr = EPI == EPI_STORE ? g.orow.off(r) + batch * g.o_bs : 0;
                                store_out<EPI, MEAN>(g, r, col, rr, split, eb[rl * 17 + cl],
                                                     eb[32 * 17 + rl * 17 + cl]);
                            }
                        }
                        __syncwarp();
                    } else if (row < g.M) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int col = n0 + cbeg + k + j;
                            if (col < g.N) store_out<EPI, MEAN>(g, row, col, ro, split, vm[j], vv[j]);
                        }
                    }
                }
            }
        }
        if (niter == 0 && row < g.M) {
            // empty reduction: outputs are the biases (or zero sums)
            for (int col = n0 + cbeg; col < min(n0 + cbeg + HC, g.N); ++col)
                store_out<EPI, MEAN>(g, row, col, ro, split, 0.f, 0.f);
        }
    }

    if (warp == R::MMA_W) {
        // The pair's MMAs read both CTAs' shared memory and write both CTAs'
        // tensor memory: wait until they are complete, also after an abort (the
        // leader commits `done` on every path out of its issue loop).
        if (!mbar_drain(done, 0) && lane == 0) atomicCAS(&g_device_error, 0, 4);
    }
    tc_fence_before();
    cluster_sync();  // no peer access (remote arrive, multicast commit) is still due
    if (warp == R::MMA_W) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(R::COLS));
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

bool tma_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = std::getenv("TAGI_B200_TMA");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Tensor maps for the raw-operand copies of a weight-sum launch whose A rows
// are contiguous along the reduction (the transposed patches) and whose B
// operands are NCHW delta planes (row map: L pixels per image, N channels, unit
// pixel stride); false (maps off) for any other operand layout. The copies
// read K-blocks of 8 reduction elements: the split reduction's chunks start on
// multiples of 8 and an image's L pixels are a multiple of 8, so a block never
// crosses an image.
// The driver's tensor-map encoder, looked up through the runtime (the library
// does not link the driver library itself); null if unavailable.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        cudaGetLastError();
    });
    return fn;
}

std::atomic<uint64_t> g_tma_launches{0};
std::atomic<uint64_t> g_tc_launches{0};

bool make_tma(const GemmArgs& g, int nc, TmaArgs* t) {
    t->on = 0;
    if (!tma_enabled() || g.bpk != nullptr || g.ga.on || g.a_bs != 0 || g.b_bs != 0) return false;
    const EncodeTiledFn encode = encode_tiled();
    if (encode == nullptr) return false;
    const int64_t L = g.brow.div;
    const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!(g.arow.div <= 0 && g.ak == 1 && g.arow.stride > 0 && (g.arow.stride * 4) % 16 == 0 &&
          al16(g.x)))
        return false;
    if (!(L > 0 && L % 8 == 0 && g.brow.stride == 1 && g.bn == L &&
          g.brow.outer == static_cast<int64_t>(g.N) * L && g.Kr % L == 0 && al16(g.u) &&
          al16(g.v) && g.kchunk % 8 == 0))
        return false;
    const int64_t rows_a = g.ones_row >= 0 ? g.ones_row : g.M;
    if (rows_a < 1) return false;
    const cuuint32_t es[3] = {1, 1, 1};
    {
        const cuuint64_t dim[2] = {static_cast<cuuint64_t>(g.Kr), static_cast<cuuint64_t>(rows_a)};
        const cuuint64_t stride[1] = {static_cast<cuuint64_t>(g.arow.stride) * 4};
        const cuuint32_t box[2] = {kBK, 128};
        if (encode(&t->a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                                   const_cast<float*>(g.x), dim, stride, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    const cuuint64_t dim[3] = {static_cast<cuuint64_t>(L), static_cast<cuuint64_t>(g.N),
                               static_cast<cuuint64_t>(g.Kr / L)};
    const cuuint64_t stride[2] = {static_cast<cuuint64_t>(L) * 4,
                                  static_cast<cuuint64_t>(g.brow.outer) * 4};
    const cuuint32_t box[3] = {kBK, static_cast<cuuint32_t>(nc), 1};
    for (int i = 0; i < 2; ++i) {
        if (encode(i ? &t->b1 : &t->b0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                                   const_cast<float*>(i ? g.v : g.u), dim, stride, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    t->L = static_cast<int>(L);
    t->on = 1;
    return true;
}

template <int VM, bool MEAN, int EPI, int BN, int GM>
int launch_tc(const GemmArgs& g, int batch, cudaStream_t st, const char* what) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    constexpr int smem = smem_bytes<VM, BN>();
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(moment_tc_kernel<VM, MEAN, EPI, BN, GM>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr_err != cudaSuccess) {
        set_error("%s: cannot reserve %d bytes of shared memory (%s)", what, smem,
                  cudaGetErrorString(attr_err));
        return TAGI_E_LAUNCH;
    }
    const int64_t pairs = (static_cast<int64_t>(g.M) + 255) / 256;
    dim3 grid(static_cast<unsigned>(2 * pairs), (g.N + BN - 1) / BN, batch * g.splits);
    TAGI_REQUIRE(grid.y <= 65535 && grid.z <= 65535, TAGI_E_UNSUPPORTED, "%s: grid too large",
                 what);
    TmaArgs tm;
    memset(&tm, 0, sizeof(tm));
    if (tma_capable<VM, BN>() && batch == 1 && make_tma(g, Roles<BN>::NC, &tm)) ++g_tma_launches;
    ++g_tc_launches;
    moment_tc_kernel<VM, MEAN, EPI, BN, GM><<<grid, Roles<BN>::THREADS, smem, st>>>(g, tm);
    return check_launch(what);
}

template <int VM, bool MEAN, int EPI, int GM = VM == FULL ? 0 : 1>
int launch_bn(const GemmArgs& g, int bn, int batch, cudaStream_t st, const char* what) {
    switch (bn) {
        case 32: return launch_tc<VM, MEAN, EPI, 32, GM>(g, batch, st, what);
        case 64: return launch_tc<VM, MEAN, EPI, 64, GM>(g, batch, st, what);
        default: return launch_tc<VM, MEAN, EPI, 128, GM>(g, batch, st, what);
    }
}

}  // namespace

int tc_pick(int vm, int M, int N, int Kr, int batch, bool fill) {
    (void)vm;
    if (!tc_enabled()) return 0;
    // Narrow operands still beat the CUDA-core kernel when the work is large
    // (the ResNet stem: reductions of 27, weight sums of 28 rows over 131072
    // pixels); the tile's unused rows and reduction elements are zero.
    if (M < 16 || N < 16 || Kr < 8) return 0;
    if (static_cast<double>(M) * N * Kr < 4.0e6) return 0;
    if (N <= 32) return 32;
    if (N <= 64 || !fill) return N <= 64 ? 64 : 128;
    // 64-column tiles halve the tensor work per staged A element, so they pay
    // only when 128-column tiles would leave more than half of the SMs idle.
    const int64_t ctas = 2 * ((static_cast<int64_t>(M) + 255) / 256) * ((N + 127) / 128) *
                         static_cast<int64_t>(batch);
    return 2 * ctas <= kNumSMs ? 64 : 128;
}

// Prepared B tiles for N tiles of 2*nc columns: column chunk cb (nc columns)
// holds, for each K-block kb, the nb tiles of that K-block exactly as a producer
// stores them in shared memory (MN-major swizzled for nc a multiple of 32, else
// K-major), so that one bulk copy moves a K-block's B side. Columns past N and
// reduction elements past Kr are zero. One thread per (chunk, K-block, 4
// columns, reduction element) in MN-major order, per (chunk, K-block, column)
// in K-major order.
template <int VM>
__global__ void pack_b_kernel(const GemmArgs g, char* dst, int nc, int nchunk, int nkb) {
    constexpr bool TWO = VM != RSQ;
    constexpr int NB = TcTiles<VM>::nb;
    const int tile = nc * 32;
    const bool mn = nc % 32 == 0;
    Side sd{};
    sd.p0 = g.u;
    sd.p1 = TWO ? g.v : g.u;
    sd.nrows = g.N;
    sd.ones_row = -1;
    const int per_kb = mn ? (nc / 4) * kBK : nc;  // threads per (chunk, K-block)
    const int64_t total = static_cast<int64_t>(nchunk) * nkb * per_kb;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t blk = i / per_kb;  // cb * nkb + kb
        const int j = static_cast<int>(i - blk * per_kb);
        const int cb = static_cast<int>(blk / nkb), kb = static_cast<int>(blk - int64_t(cb) * nkb);
        char* st = dst + blk * NB * tile;
        if (mn) {
            const int r = (j % (nc / 4)) * 4, k = j / (nc / 4);
            float x[4], y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (kb * kBK + k < g.Kr)
                    load_elem<false, TWO>(g, sd, cb * nc + r + e, kb * kBK + k, x[e], y[e]);
                else
                    x[e] = y[e] = 0.f;
            }
            store_tiles<VM, false>(st, tile, tile_off_mn(r, k, nc), x, y);
        } else {
            const int row = cb * nc + j;
            const int64_t base = row < g.N ? row_base<false>(g, row) : 0;
            float v[2][8];
            load_row<false, TWO, 0>(g, sd, row, base, GatherRow{0, 0, 0}, kb * kBK, g.Kr, v);
            store_tiles<VM, false>(st, tile, tile_off_k(j, 0), &v[0][0], &v[1][0]);
            store_tiles<VM, false>(st, tile, tile_off_k(j, 4), &v[0][4], &v[1][4]);
        }
    }
}

size_t tc_pack_bytes(int vm, int N, int Kr, int bn) {
    if (N <= 0 || Kr <= 0 || bn <= 0) return 0;
    const int64_t cols = (static_cast<int64_t>(N) + bn - 1) / bn * bn;
    const int64_t nkb = (static_cast<int64_t>(Kr) + kBK - 1) / kBK;
    const int nb = vm == FULL ? TcTiles<FULL>::nb : TcTiles<RSQ>::nb;  // LSQ: as RSQ
    return static_cast<size_t>(nkb * nb * cols * 32);
}

int tc_pack_b(GemmArgs& g, int vm, int bn, void* dst, cudaStream_t st, const char* what) {
    TAGI_REQUIRE(vm == FULL || vm == RSQ || vm == LSQ, TAGI_E_UNSUPPORTED,
                 "%s: no prepared B for mode %d", what, vm);
    TAGI_REQUIRE(bn == 32 || bn == 64 || bn == 128, TAGI_E_UNSUPPORTED, "%s: N tile %d", what, bn);
    TAGI_REQUIRE((reinterpret_cast<uintptr_t>(dst) & 255) == 0, TAGI_E_ALIGNMENT,
                 "%s: prepared-B buffer not 256-byte aligned", what);
    const int nc = bn / 2, nchunk = (g.N + bn - 1) / bn * 2, nkb = (g.Kr + kBK - 1) / kBK;
    const int64_t per_kb = nc % 32 == 0 ? (nc / 4) * kBK : nc;
    const int64_t total = static_cast<int64_t>(nchunk) * nkb * per_kb;
    if (total > 0) {
        char* d = static_cast<char*>(dst);
        if (vm == FULL)
            pack_b_kernel<FULL><<<grid_1d(total, 256), 256, 0, st>>>(g, d, nc, nchunk, nkb);
        else if (vm == RSQ)
            pack_b_kernel<RSQ><<<grid_1d(total, 256), 256, 0, st>>>(g, d, nc, nchunk, nkb);
        else
            pack_b_kernel<LSQ><<<grid_1d(total, 256), 256, 0, st>>>(g, d, nc, nchunk, nkb);
        const int rc = check_launch(what);
        if (rc) return rc;
    }
    g.bpk = static_cast<const char*>(dst);
    g.bpk_nc = nc;
    g.bpk_nkb = nkb;
    return TAGI_OK;
}

int tc_launch(const GemmArgs& g, int vm, bool mean, int epi, int bn, int batch, cudaStream_t st,
              const char* what) {
    if (g.M == 0 || g.N == 0) return TAGI_OK;
    if (vm == FULL) {
        if (epi == EPI_PARTIAL && mean) return launch_bn<FULL, true, EPI_PARTIAL>(g, bn, batch, st, what);
        if (epi != EPI_STORE) return TAGI_E_UNSUPPORTED;
        return mean ? launch_bn<FULL, true, EPI_STORE>(g, bn, batch, st, what)
                    : launch_bn<FULL, false, EPI_STORE>(g, bn, batch, st, what);
    }
    if (vm == RSQ) {
        if ((epi != EPI_STORE && epi != EPI_PARTIAL) || !mean) return TAGI_E_UNSUPPORTED;
        // the stride-1 col2im gather compiles without divisions
        const bool s1 = g.ga.on && g.ga.s == 1;
        if (epi == EPI_PARTIAL)
            return s1 ? launch_bn<RSQ, true, EPI_PARTIAL, 2>(g, bn, batch, st, what)
                      : launch_bn<RSQ, true, EPI_PARTIAL, 1>(g, bn, batch, st, what);
        return s1 ? launch_bn<RSQ, true, EPI_STORE, 2>(g, bn, batch, st, what)
                  : launch_bn<RSQ, true, EPI_STORE, 1>(g, bn, batch, st, what);
    }
    if (!mean) return TAGI_E_UNSUPPORTED;
    switch (epi) {
        case EPI_STORE: return launch_bn<LSQ, true, EPI_STORE>(g, bn, batch, st, what);
        case EPI_PARTIAL: return launch_bn<LSQ, true, EPI_PARTIAL>(g, bn, batch, st, what);
        default: return launch_bn<LSQ, true, EPI_PARAM>(g, bn, batch, st, what);
    }
}

}  // namespace tagi

extern "C" uint64_t tagi_tma_launches(void) { return tagi::g_tma_launches.load(); }
extern "C" uint64_t tagi_tc_launches(void) { return tagi::g_tc_launches.load(); }

extern "C" int tagi_set_wait_limit_ns(uint64_t ns) {
    const unsigned long long v = ns ? static_cast<unsigned long long>(ns) : tagi::kTimeoutNs;
    const int force = (ns > 0 && ns < 1000) ? 1 : 0;
    cudaError_t e = cudaMemcpyToSymbol(tagi::g_wait_limit_ns, &v, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(tagi::g_force_abort, &force, sizeof(force));
    if (e != cudaSuccess) {
        cudaGetLastError();
        tagi::set_error("tagi_set_wait_limit_ns: %s", cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    return TAGI_OK;
}

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
