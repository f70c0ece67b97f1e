// runtime.h -- host-side runtime of libx100gemm_b200.so: per-device context
// (stream, status word, grow-only staging buffers, tensor-map encoder),
// thread-local error reporting, pointer classification and the host-side
// fault injector.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <mutex>

#include "../../include/x100_gemm.h"

namespace x100 {

// Per-thread status of the last API call.
void set_error(int code);
int get_error();

// X100_FAULT=<site>[,<site>...] makes the library fail at that site without
// touching the GPU: "alloc", "copy", "launch", "device", "comm".  Returns
// true (and records X100_E_INJECTED) when the site is armed.
bool fault_injected(const char *site);

// A grow-only device buffer owned by a context.
struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
};

struct DevCtx {
    int device = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    size_t smem_optin = 0;
    cudaStream_t stream = nullptr;   // stream of the synchronous host-pointer API
    int *d_status = nullptr;         // device status word written by kernels
    DevBuf stage[6];                 // staging buffers of host-pointer calls
    std::mutex mu;                   // serialises host-pointer calls on this device
    // Panelled host-pointer calls: host->device copies on `up`, device->host
    // copies on `down`, the kernels on `stream`; ev[p] marks panel p's inputs
    // staged, ev[kMaxPanels + p] panel p computed.
    // ev[2 * kMaxPanels] marks B staged.
    static constexpr int kMaxPanels = 8;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev[2 * kMaxPanels + 1] = {};
    // Stream-ordered scratch of kernels that need temporaries (the tf32
    // split operands): a pool of the library's own that keeps up to
    // kPoolKeepBytes mapped across synchronisations, so a call after a sync
    // does not map its scratch again.
    static constexpr uint64_t kPoolKeepBytes = 4ull << 30;
    cudaMemPool_t pool = nullptr;
};

// Context of the calling thread's selected device (created on first use).
// Returns nullptr and records the error if no usable device exists.
DevCtx *ctx();
int current_device();
// Makes `device` current for the guard's lifetime and restores the caller's
// current device afterwards (used where the library frees memory it owns).
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            cudaGetLastError();
            prev = -1;
        }
        if (prev != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Ensure staging buffer `slot` of `c` holds at least `bytes`; returns its
// device pointer or nullptr (error recorded).
void *stage_buf(DevCtx *c, int slot, size_t bytes);

// True when `p` is device (or managed) memory usable by kernels directly.
bool is_device_ptr(const void *p);

// Encode a 2-D row-major tensor map: `inner` elements per row (contiguous),
// `outer` rows, `row_stride_bytes` between rows, box `box_inner` x
// `box_outer`, 128-byte swizzle, out-of-bounds elements read as zero.
bool make_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
// The same with the swizzle chosen by the caller (CU_TENSOR_MAP_SWIZZLE_NONE
// for plain row-by-row boxes).
bool make_tmap_2d_sw(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);

// Map a CUDA error to an X100 status and record it.  Returns the status.
int check_cuda(cudaError_t e, int code_if_error);

// Read and clear the device status word after synchronising `s`.
int sync_and_status(DevCtx *c, cudaStream_t s);

}  // namespace x100
