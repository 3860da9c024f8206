// Small all-reduces over NVLink peer memory: the SyncBN statistics exchange.
//
// A data-parallel BatchNorm2D all-reduces 3*C float64 channel sums (a few KB)
// before it can normalise, twenty times per ResNet-18 step, each on the
// critical path; a library all-reduce spends tens of microseconds on such a
// message. Here every rank owns one buffer of identical layout (allocated by
// tagi_peer_buffer_create, exported with a CUDA IPC handle, opened by every
// other rank):
//   [0, 256)   one flag per source rank (uint64 epochs; 32 ranks at most)
//   [256, ...) two parity sets x world slots x max_elems doubles
// One kernel per all-reduce: each rank stores its values into slot [rank] of
// the current parity set in every rank's buffer (plain peer stores, no
// multicast), publishes its epoch in every rank's flag [rank] with a
// system-scope release, waits (bounded) until all flags of its own buffer
// reached the epoch, and adds the slots in rank order, so every rank computes
// bit-identical sums. The epoch is a device counter that the kernel advances,
// so the same launch can be replayed from a CUDA graph; all ranks must issue
// the same sequence of exchanges.
//
// Slot reuse: a rank writes parity set p of epoch e + 2 only after its own
// exchange e + 1 completed, which needed every peer's flag e + 1, which a peer
// publishes only after its exchange e (its read of set p) finished in stream
// order. Two sets therefore suffice.
//
// Waits are bounded (2 s): on timeout the kernel records the error word read
// by tagi_peer_status, leaves the data unreduced and returns.
#include <cstring>

#include "common.cuh"

namespace tagi {

__device__ int g_peer_error = 0;

namespace {

constexpr int kMaxRanks = 32;
constexpr size_t kFlagBytes = 256;
constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;

__device__ __forceinline__ unsigned long long peer_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(256) peer_allreduce_kernel(double* data, int n,
                                                             char* const* bufs, int rank,
                                                             int world, int max_elems,
                                                             unsigned long long* counter) {
    __shared__ unsigned long long s_epoch;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_epoch = *counter + 1;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned long long epoch = s_epoch;
    const int parity = static_cast<int>(epoch & 1ull);
    const size_t set_elems = static_cast<size_t>(world) * max_elems;
    // 1. my values into slot [rank] of every rank's buffer
    for (int p = 0; p < world; ++p) {
        double* slot = reinterpret_cast<double*>(bufs[p] + kFlagBytes) + parity * set_elems +
                       static_cast<size_t>(rank) * max_elems;
        for (int i = threadIdx.x; i < n; i += blockDim.x) slot[i] = data[i];
    }
    __threadfence_system();
    __syncthreads();
    // 2. publish the epoch in flag [rank] of every buffer
    if (threadIdx.x < world) {
        unsigned long long* flag =
            reinterpret_cast<unsigned long long*>(bufs[threadIdx.x]) + rank;
        st_release_sys(flag, epoch);
    }
    // 3. wait for every rank's flag in my buffer
    if (threadIdx.x < world) {
        const unsigned long long* flag =
            reinterpret_cast<const unsigned long long*>(bufs[rank]) + threadIdx.x;
        const unsigned long long t0 = peer_timer();
        while (ld_acquire_sys(flag) < epoch) {
            if (peer_timer() - t0 > kPeerTimeoutNs) {
                atomicCAS(&g_peer_error, 0, 1);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;  // the counter stays, so the ranks' epochs disagree from here on
    // 4. sum the slots of my buffer in rank order
    const double* mine = reinterpret_cast<const double*>(bufs[rank] + kFlagBytes) +
                         parity * set_elems;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        double s = 0.0;
        for (int r = 0; r < world; ++r) s += mine[static_cast<size_t>(r) * max_elems + i];
        data[i] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = epoch;
}

}  // namespace
}  // namespace tagi

using namespace tagi;

extern "C" size_t tagi_peer_buffer_bytes(int world, int64_t max_elems) {
    if (world < 1 || world > kMaxRanks || max_elems < 1) return 0;
    return kFlagBytes + 2ull * static_cast<size_t>(world) * static_cast<size_t>(max_elems) *
                            sizeof(double);
}

extern "C" int tagi_peer_buffer_create(size_t bytes, void** ptr, void* ipc_handle) {
    const char* what = "tagi_peer_buffer_create";
    TAGI_REQUIRE(bytes >= kFlagBytes && ptr && ipc_handle, TAGI_E_BAD_ARG, "%s: bad arguments",
                 what);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (p) cudaFree(p);
        set_error("%s: %s", what, cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return TAGI_OK;
}

extern "C" int tagi_peer_buffer_open(const void* ipc_handle, void** ptr) {
    const char* what = "tagi_peer_buffer_open";
    TAGI_REQUIRE(ipc_handle && ptr, TAGI_E_BAD_ARG, "%s: bad arguments", what);
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: %s", what, cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    *ptr = p;
    return TAGI_OK;
}

extern "C" int tagi_peer_buffer_close(void* ptr, int own) {
    if (ptr == nullptr) return TAGI_OK;
    const cudaError_t e = own ? cudaFree(ptr) : cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("tagi_peer_buffer_close: %s", cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    return TAGI_OK;
}

extern "C" int tagi_peer_allreduce_f64(double* data, int64_t n, void* const* peer_bufs, int rank,
                                       int world, int64_t max_elems, uint64_t* counter,
                                       void* stream) {
    const char* what = "tagi_peer_allreduce_f64";
    TAGI_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world && n >= 0 &&
                     n <= max_elems && max_elems <= (int64_t(1) << 28),
                 TAGI_E_BAD_ARG, "%s: bad sizes", what);
    TAGI_REQUIRE(data && peer_bufs && counter, TAGI_E_BAD_ARG, "%s: null pointer", what);
    peer_allreduce_kernel<<<1, 256, 0, as_stream(stream)>>>(
        data, static_cast<int>(n), reinterpret_cast<char* const*>(peer_bufs), rank, world,
        static_cast<int>(max_elems), reinterpret_cast<unsigned long long*>(counter));
    return check_launch(what);
}

extern "C" int tagi_peer_status(int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, tagi::g_peer_error, sizeof(int));
    if (e != cudaSuccess) {
        cudaGetLastError();
        tagi::set_error("tagi_peer_status: %s", cudaGetErrorString(e));
        return TAGI_E_LAUNCH;
    }
    if (reset && v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(tagi::g_peer_error, &zero, sizeof(int));
    }
    return v;
}
