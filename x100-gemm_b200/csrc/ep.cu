// ep.cu -- the expert-parallel combine: a one-shot all-reduce of the experts'
// partial outputs over peer memory (NVLink), and the x100q_ep_* entry points
// of include/x100q.h.
//
// In the reference the MoE block runs on one process (qwen_moe.c:305-310);
// with experts split over G processes (x100q_moe_create(lo, hi)) each holds a
// partial eout that must be summed.  Each process owns one device buffer
// (exported with cudaIpcGetMemHandle, opened by the others):
//   recv  [2 parities][G sources][cap] floats
//   flags [2 parities][G sources][kEpCtas] u32 epoch stamps
//   epoch [kEpCtas] u32, this process's completed combines per CTA slot
// Call e (1, 2, ...) of CTA c, parity e & 1: the CTA stores its slice of the
// local partial into recv[par][rank] of every process (plain stores, its own
// included), then one thread publishes flags[par][rank][c] = e on every
// process (a release at system scope); it then waits
// (bounded) until every source's flag for slice c reads e, and sums the G
// slices in source order -- the same order on every process, so all of them
// end with identical bits.  A source can be at most one call ahead (it waits
// for everyone's call e before starting e + 1), so two parities keep a slot
// from being overwritten while it is read.  Peer memory is only ever reached
// by plain loads and stores.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/x100q.h"
#include "ptx.cuh"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace ep {

constexpr int kEpMax = 8;         // processes
constexpr int kEpCtas = 32;       // CTA slots (slices) per call
constexpr int kEpThreads = 256;
constexpr unsigned long long kEpWaitNs = 1000000000ull;   // 1 s

struct Peers {
    uint8_t *base[kEpMax];
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// grid: G <= kEpCtas CTAs, slice c = [c * chunk, min(n, (c+1) * chunk)).
__global__ void __launch_bounds__(kEpThreads)
    ep_allreduce_kernel(const Peers peers, int rank, int world, long cap, const float *__restrict__ src,
                        float *__restrict__ dst, int n, int chunk, int accum, int *status) {
    const int c = blockIdx.x;
    uint8_t *mine = peers.base[rank];
    float *recv = reinterpret_cast<float *>(mine);
    uint32_t *flags = reinterpret_cast<uint32_t *>(mine + 2 * (size_t)kEpMax * cap * 4);
    uint32_t *epoch = flags + 2 * kEpMax * kEpCtas;
    __shared__ uint32_t s_e;
    __shared__ int s_timeout;
    q::pdl_launch_dependents();
    q::pdl_wait();   // src comes from the previous kernel; every earlier call of this slot has completed
    if (threadIdx.x == 0) {
        s_e = epoch[c] + 1;   // read after the wait: the previous call may run until then
        s_timeout = 0;
    }
    __syncthreads();
    const uint32_t e = s_e;
    const int par = e & 1;
    const int i0 = c * chunk, i1 = min(n, i0 + chunk);
    // 1. my slice of the partial into recv[par][rank] of every process
    for (int p = 0; p < world; ++p) {
        float *d = reinterpret_cast<float *>(peers.base[p]) + ((size_t)par * kEpMax + rank) * cap;
        for (int i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x)
            *reinterpret_cast<float4 *>(d + i) = __ldcg(reinterpret_cast<const float4 *>(src + i));
    }
    __syncthreads();
    // 2. publish: flag[par][rank][c] = e on every process (a system-scope
    // release: the CTA's stores above, ordered before it by the barrier,
    // become visible to a peer that acquires the flag)
    if (threadIdx.x < world) {
        uint32_t *f = reinterpret_cast<uint32_t *>(peers.base[threadIdx.x] + 2 * (size_t)kEpMax * cap * 4);
        st_release_sys(f + ((size_t)par * kEpMax + rank) * kEpCtas + c, e);
    }
    // 3. wait for every source's slice c of call e (bounded)
    if (threadIdx.x < world) {
        const uint32_t *f = flags + ((size_t)par * kEpMax + threadIdx.x) * kEpCtas + c;
        const unsigned long long t0 = globaltimer_ns();
        while (ld_acquire_sys(f) != e) {
            if (globaltimer_ns() - t0 > kEpWaitNs) {
                s_timeout = 1;
                atomicCAS(status, 0, X100_E_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
    // 4. sum the sources in order
    if (!s_timeout) {
        for (int i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x) {
            float4 t = accum ? *reinterpret_cast<const float4 *>(dst + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < world; ++r) {
                const float4 v = __ldcg(reinterpret_cast<const float4 *>(recv + ((size_t)par * kEpMax + r) * cap + i));
                t.x += v.x;
                t.y += v.y;
                t.z += v.z;
                t.w += v.w;
            }
            *reinterpret_cast<float4 *>(dst + i) = t;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) epoch[c] = e;
}

}  // namespace ep
}  // namespace x100

using namespace x100;
using namespace x100::ep;

struct x100q_ep {
    int device = 0, world = 1, rank = 0;
    long cap = 0;                 // floats per source slot
    size_t bytes = 0;
    uint8_t *buf = nullptr;       // this process's buffer
    Peers peers;
    bool opened = false;
    cudaIpcMemHandle_t handle;
};

static_assert(sizeof(cudaIpcMemHandle_t) == X100Q_EP_HANDLE_BYTES, "IPC handle size");

extern "C" {

x100q_ep *x100q_ep_create(int world, int rank, int max_floats) {
    set_error(X100_OK);
    if (world < 1 || world > kEpMax || rank < 0 || rank >= world || max_floats <= 0 || max_floats % 4) {
        set_error(X100_E_ARG);
        return nullptr;
    }
    DevCtx *c = ctx();
    if (!c) return nullptr;
    if (fault_injected("alloc")) return nullptr;
    x100q_ep *e = new x100q_ep();
    e->device = c->device;
    e->world = world;
    e->rank = rank;
    e->cap = max_floats;
    e->bytes = 2 * (size_t)kEpMax * max_floats * 4 + 2 * (size_t)kEpMax * kEpCtas * 4 + (size_t)kEpCtas * 4;
    if (cudaMalloc(&e->buf, e->bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        delete e;
        return nullptr;
    }
    if (check_cuda(cudaMemset(e->buf, 0, e->bytes), X100_E_ALLOC) ||
        check_cuda(cudaIpcGetMemHandle(&e->handle, e->buf), X100_E_COMM) ||
        check_cuda(cudaDeviceSynchronize(), X100_E_ALLOC)) {
        cudaFree(e->buf);
        delete e;
        return nullptr;
    }
    for (int p = 0; p < kEpMax; ++p) e->peers.base[p] = nullptr;
    e->peers.base[rank] = e->buf;
    return e;
}

int x100q_ep_handle(const x100q_ep *e, void *handle_out) {
    if (!e || !handle_out) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    memcpy(handle_out, &e->handle, X100Q_EP_HANDLE_BYTES);
    return X100_OK;
}

int x100q_ep_open(x100q_ep *e, const void *all_handles) {
    set_error(X100_OK);
    if (!e || !all_handles || e->opened) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(e->device);
    if (fault_injected("comm")) return X100_E_INJECTED;
    const uint8_t *h = static_cast<const uint8_t *>(all_handles);
    for (int p = 0; p < e->world; ++p) {
        if (p == e->rank) continue;
        cudaIpcMemHandle_t hp;
        memcpy(&hp, h + (size_t)p * X100Q_EP_HANDLE_BYTES, X100Q_EP_HANDLE_BYTES);
        void *ptr = nullptr;
        if (check_cuda(cudaIpcOpenMemHandle(&ptr, hp, cudaIpcMemLazyEnablePeerAccess), X100_E_COMM)) {
            for (int q = 0; q < p; ++q)
                if (q != e->rank && e->peers.base[q]) cudaIpcCloseMemHandle(e->peers.base[q]);
            return X100_E_COMM;
        }
        e->peers.base[p] = static_cast<uint8_t *>(ptr);
    }
    e->opened = true;
    return X100_OK;
}

int x100q_ep_allreduce_dev(x100q_ep *e, const float *src, float *dst, int n, int accum, void *stream) {
    set_error(X100_OK);
    if (!e || !e->opened || !src || !dst || n <= 0 || n % 4 || n > e->cap ||
        (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15)) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    // slices of at least 1024 floats, at most kEpCtas of them; the same n gives
    // the same split on every process
    int g = (n + 1023) / 1024;
    if (g > kEpCtas) g = kEpCtas;
    const int chunk = ((n + g - 1) / g + 3) & ~3;
    g = (n + chunk - 1) / chunk;
    const int st = launch_pdl(ep_allreduce_kernel, dim3(g), dim3(kEpThreads), 0, static_cast<cudaStream_t>(stream),
                              e->peers, e->rank, e->world, e->cap, src, dst, n, chunk, accum, c->d_status);
    if (st) set_error(st);
    return st;
}

void x100q_ep_destroy(x100q_ep *e) {
    if (!e) return;
    DeviceGuard dg(e->device);
    if (e->opened)
        for (int p = 0; p < e->world; ++p)
            if (p != e->rank && e->peers.base[p]) cudaIpcCloseMemHandle(e->peers.base[p]);
    cudaFree(e->buf);
    delete e;
}

}  // extern "C"
