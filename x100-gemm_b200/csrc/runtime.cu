// runtime.cu -- per-device contexts, errors, tensor maps, pointer
// classification, fault injection and capability detection.
#include "runtime.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace x100 {

static thread_local int t_error = 0;
// Device chosen with x100_set_device on this thread, or -1: follow the
// thread's current CUDA device (one process or thread per GPU).
static thread_local int t_device = -1;

void set_error(int code) { t_error = code; }
int get_error() { return t_error; }

bool fault_injected(const char *site) {
    const char *f = getenv("X100_FAULT");
    if (!f || !*f) return false;
    size_t n = strlen(site);
    for (const char *p = f; (p = strstr(p, site)) != nullptr; p += n) {
        bool lb = (p == f) || p[-1] == ',';
        bool rb = p[n] == '\0' || p[n] == ',';
        if (lb && rb) {
            set_error(X100_E_INJECTED);
            return true;
        }
    }
    return false;
}

int check_cuda(cudaError_t e, int code_if_error) {
    if (e == cudaSuccess) return X100_OK;
    set_error(code_if_error);
    if (getenv("X100_VERBOSE")) fprintf(stderr, "[x100] CUDA error %d: %s\n", (int)e, cudaGetErrorString(e));
    return code_if_error;
}

static std::mutex g_ctx_mu;
static DevCtx *g_ctx[64];

int current_device() {
    if (t_device >= 0) return t_device;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        d = 0;
    }
    return d;
}

DevCtx *ctx() {
    if (fault_injected("device")) return nullptr;
    const int dev = current_device();
    if (dev < 0 || dev >= 64) {
        set_error(X100_E_ARG);
        return nullptr;
    }
    {
        std::lock_guard<std::mutex> lk(g_ctx_mu);
        if (g_ctx[dev]) {
            if (t_device >= 0) cudaSetDevice(dev);   // explicit choice; otherwise dev is already current
            return g_ctx[dev];
        }
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= dev) {
            cudaGetLastError();
            set_error(X100_E_NODEV);
            return nullptr;
        }
        if (cudaSetDevice(dev) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_NODEV);
            return nullptr;
        }
        DevCtx *c = new DevCtx();
        c->device = dev;
        cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&c->cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&c->cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        c->smem_optin = (size_t)optin;
        bool ok = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&c->up, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&c->down, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaMalloc(&c->d_status, 64) == cudaSuccess && cudaMemset(c->d_status, 0, 64) == cudaSuccess;
        for (cudaEvent_t &e : c->ev) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
        if (ok) {
            cudaMemPoolProps pp = {};
            pp.allocType = cudaMemAllocationTypePinned;
            pp.location.type = cudaMemLocationTypeDevice;
            pp.location.id = dev;
            uint64_t keep = DevCtx::kPoolKeepBytes;
            ok = cudaMemPoolCreate(&c->pool, &pp) == cudaSuccess &&
                 cudaMemPoolSetAttribute(c->pool, cudaMemPoolAttrReleaseThreshold, &keep) == cudaSuccess;
        }
        if (!ok) {
            cudaGetLastError();
            delete c;
            set_error(X100_E_ALLOC);
            return nullptr;
        }
        g_ctx[dev] = c;
        return c;
    }
}

void *stage_buf(DevCtx *c, int slot, size_t bytes) {
    if (fault_injected("alloc")) return nullptr;
    DevBuf &b = c->stage[slot];
    if (b.bytes >= bytes && b.ptr) return b.ptr;
    if (b.ptr) {
        cudaStreamSynchronize(c->stream);
        cudaFree(b.ptr);
        b.ptr = nullptr;
        b.bytes = 0;
    }
    size_t want = bytes < 256 ? 256 : bytes;
    if (cudaMalloc(&b.ptr, want) != cudaSuccess) {
        cudaGetLastError();
        b.ptr = nullptr;
        set_error(X100_E_ALLOC);
        return nullptr;
    }
    b.bytes = want;
    return b.ptr;
}

bool is_device_ptr(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

static PFN_encodeTiled encoder() {
    static PFN_encodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

bool make_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
    return make_tmap_2d_sw(m, base, dt, inner, outer, row_stride_bytes, box_inner, box_outer,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

bool make_tmap_2d_sw(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                     uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    PFN_encodeTiled enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int sync_and_status(DevCtx *c, cudaStream_t s) {
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return check_cuda(e, X100_E_LAUNCH);
    int st = 0;
    e = cudaMemcpy(&st, c->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return check_cuda(e, X100_E_LAUNCH);
    if (st) {
        cudaMemset(c->d_status, 0, sizeof(int));
        set_error(st);
    }
    return st;
}

}  // namespace x100

using namespace x100;

extern "C" {

int x100_last_error(void) { return get_error(); }

const char *x100_strerror(int code) {
    switch (code) {
    case X100_OK: return "ok";
    case X100_E_ARG: return "invalid argument";
    case X100_E_NODEV: return "no usable CUDA device";
    case X100_E_ARCH: return "device is not sm_100 (B200); the tcgen05 path needs compute capability 10.x";
    case X100_E_ALLOC: return "device or pinned memory allocation failed";
    case X100_E_COPY: return "host<->device copy failed";
    case X100_E_LAUNCH: return "kernel launch or execution failed";
    case X100_E_TIMEOUT: return "a device-side wait hit its iteration limit";
    case X100_E_COMM: return "collective / peer exchange failed";
    case X100_E_INJECTED: return "failure injected by X100_FAULT";
    case X100_E_UNSUPPORTED: return "unsupported shape, type or layout";
    case X100_E_TOO_LARGE:
        return "request larger than the fixed scratch of a no-allocation entry point";
    case X100_E_FORMAT: return "malformed file, or a tensor missing or of a type that cannot be used";
    default: return "unknown error";
    }
}

int x100_set_device(int device) {
    if (device < 0 || device >= 64) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    t_device = device;
    set_error(X100_OK);
    return X100_OK;
}

int x100_sync(void *stream) {
    DevCtx *c = ctx();
    if (!c) return get_error();
    set_error(X100_OK);
    return sync_and_status(c, (cudaStream_t)stream);
}

// replaces x100_detect (reference src/x100_caps.c:24-62): fills the same
// struct from the CUDA device instead of /proc/cpuinfo.
void x100_detect(x100_caps_t *caps) {
    if (!caps) return;
    memset(caps, 0, sizeof(*caps));
    caps->mvendorid = 0x10de;
    DevCtx *c = ctx();
    if (!c) {
        snprintf(caps->isa, sizeof(caps->isa), "no CUDA device (%s)", x100_strerror(get_error()));
        return;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, c->device) != cudaSuccess) {
        cudaGetLastError();
        snprintf(caps->isa, sizeof(caps->isa), "cuda device %d (properties unavailable)", c->device);
        return;
    }
    caps->has_zvfh = 1;
    caps->has_ime = (c->cc_major == 10) ? 1 : 0;
    snprintf(caps->isa, sizeof(caps->isa), "%s sm_%d%d %d SMs %zu MiB HBM, tcgen05=%s, smem/block %zu KiB", p.name,
             c->cc_major, c->cc_minor, c->sm_count, (size_t)(p.totalGlobalMem >> 20),
             caps->has_ime ? "yes" : "no", c->smem_optin >> 10);
    set_error(X100_OK);
}

// replaces x100_caps_print (reference src/x100_caps.c:64-76)
void x100_caps_print(const x100_caps_t *c) {
    if (!c) return;
    printf("== x100 capabilities (CUDA) ==\n");
    printf("  mvendorid : 0x%lx %s\n", c->mvendorid, c->mvendorid == 0x10de ? "(NVIDIA)" : "");
    printf("  fp16 GEMM : %s\n", c->has_zvfh ? "yes" : "no");
    printf("  tcgen05   : %s  (int8/fp16 tensor-core GEMM)\n", c->has_ime ? "yes" : "no");
    printf("  device    : %.200s\n", c->isa);
}

}  // extern "C"
