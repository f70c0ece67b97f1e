// x100_gemm_shim.cu -- the extern "C" entry points of include/x100_gemm.h.
//
// Host-pointer calls (the reference's own signatures) stage operands into
// grow-only device buffers (padding leading dimensions to 16 bytes so the
// tensor-core path's TMA maps are legal), run the kernel on the context's
// stream and copy C back before returning; calls that move 32 MiB or more of
// host A and C run as row panels whose copies in, kernels and copies out
// overlap.  Device pointers are detected and used in place.  Every failure is recorded for x100_last_error(); nothing
// aborts.
#include <cuda_fp16.h>

#include <cstring>

#include "gemm_kernels.h"

using namespace x100;

namespace {

long round_up(long v, long a) { return (v + a - 1) / a * a; }

// Device view of an operand: either the caller's device memory or a staged
// copy with a padded leading dimension.
struct Operand {
    const void *dev = nullptr;
    long ld = 0;
};

// Stage a rows x cols row-major host/device matrix (element size es) into
// staging slot `slot` with its leading dimension padded to `pad_elems`,
// unless it is device memory that already satisfies the alignment.
bool stage_in(DevCtx *c, int slot, const void *p, long rows, long cols, int es, long pad_elems, bool need_align,
              Operand &out, cudaStream_t s) {
    const bool dev = is_device_ptr(p);
    const bool aligned = (reinterpret_cast<uintptr_t>(p) % 16 == 0) && ((cols * es) % 16 == 0);
    if (dev && (!need_align || aligned)) {
        out.dev = p;
        out.ld = cols;
        return true;
    }
    const long ld = need_align ? round_up(cols, pad_elems) : cols;
    void *d = stage_buf(c, slot, (size_t)(ld * rows * es));
    if (!d) return false;
    if (fault_injected("copy")) return false;
    cudaError_t e = cudaMemcpy2DAsync(d, ld * es, p, cols * es, cols * es, rows,
                                      dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        check_cuda(e, X100_E_COPY);
        return false;
    }
    out.dev = d;
    out.ld = ld;
    return true;
}

// C operand (read-modify-write): used in place when on the device, else
// staged in and copied back after the kernel.
struct COperand {
    void *dev = nullptr;
    void *host = nullptr;
    size_t bytes = 0;
};

bool stage_c(DevCtx *c, int slot, void *p, size_t bytes, bool load, COperand &out) {
    if (is_device_ptr(p)) {
        out.dev = p;
        return true;
    }
    void *d = stage_buf(c, slot, bytes);
    if (!d) return false;
    if (fault_injected("copy")) return false;
    if (load) {
        cudaError_t e = cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, c->stream);
        if (e != cudaSuccess) {
            check_cuda(e, X100_E_COPY);
            return false;
        }
    }
    out.dev = d;
    out.host = p;
    out.bytes = bytes;
    return true;
}

int finish_c(DevCtx *c, const COperand &co) {
    if (co.host) {
        cudaError_t e = cudaMemcpyAsync(co.host, co.dev, co.bytes, cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) return check_cuda(e, X100_E_COPY);
    }
    return sync_and_status(c, c->stream);
}

bool dims_ok(int M, int N, int K, const void *A, const void *B, const void *C) {
    if (M < 0 || N < 0 || K < 0 || (M > 0 && N > 0 && K > 0 && (!A || !B || !C))) {
        set_error(X100_E_ARG);
        return false;
    }
    return true;
}

enum Route { ROUTE_TC_I8, ROUTE_SIMT_I8, ROUTE_F32_FAST, ROUTE_F32_REF, ROUTE_F16_F32C, ROUTE_F16_F16C };

// The fast fp32 GEMM: three tf32 tensor-core products (A_hi.B_hi + A_hi.B_lo +
// A_lo.B_hi, relative error about 1e-6, inside the 1e-5 bar) when TMA can
// address the operands and CTA pairs can be scheduled, else the FFMA kernel.
// X100_GEMM_F32_FFMA=1 keeps the FFMA kernel.
int f32_fast(DevCtx *c, int M, int N, int K, const float *A, long lda, const float *B, long ldb, float *C, long ldc,
             cudaStream_t s) {
    static const bool ffma = getenv("X100_GEMM_F32_FFMA") != nullptr;
    if (!ffma && tc_operands_ok(3, A, lda, B, ldb)) {
        const int st = launch_gemm_tc(c, 3, M, N, K, A, lda, B, ldb, C, ldc, s);
        if (st != X100_E_UNSUPPORTED) return st;
        set_error(X100_OK);
    }
    return launch_gemm_f32_fast(c, M, N, K, A, lda, B, ldb, C, ldc, s);
}

// Launch `route`'s kernel for C (M x N, ld ldc) += A (M x K) . B (K x N) on s.
int launch_route(DevCtx *c, Route route, int M, int N, int K, const void *A, long lda, const void *B, long ldb,
                 void *C, long ldc, cudaStream_t s) {
    switch (route) {
    case ROUTE_TC_I8: return launch_gemm_tc(c, 0, M, N, K, A, lda, B, ldb, C, ldc, s);
    case ROUTE_SIMT_I8:
        return launch_gemm_i8_simt(c, M, N, K, (const int8_t *)A, lda, (const int8_t *)B, ldb, (int32_t *)C, ldc, s);
    case ROUTE_F32_FAST:
        return f32_fast(c, M, N, K, (const float *)A, lda, (const float *)B, ldb, (float *)C, ldc, s);
    case ROUTE_F32_REF:
        return launch_gemm_f32_ref(c, M, N, K, (const float *)A, lda, (const float *)B, ldb, (float *)C, ldc, s);
    case ROUTE_F16_F32C: return launch_gemm_tc(c, 1, M, N, K, A, lda, B, ldb, C, ldc, s);
    case ROUTE_F16_F16C: return launch_gemm_tc(c, 2, M, N, K, A, lda, B, ldb, C, ldc, s);
    }
    return X100_E_ARG;
}

// Rows of C per panel of a panelled host call: a multiple of the 256-row
// tile, at most DevCtx::kMaxPanels panels.
constexpr long kPanelAlign = 256;
// Host calls moving fewer bytes than this run as one copy-in, kernel, copy-out.
constexpr size_t kPanelMinBytes = 32u << 20;

// Host A and host C: the call runs as row panels so that the three engines
// overlap.  On `up`: B (whole), then per panel its rows of A and of C; on
// `stream`: panel p's kernel once ev[p] says its rows arrived; on `down`:
// panel p's rows of C back once ev[kMaxPanels + p] says they are final.
// Each row of C depends only on its row of A and on B, so the panels are the
// whole product; the host->device and device->host copies run at the same
// time (PCIe is full duplex) and the kernels hide behind them.
int host_gemm_panels(DevCtx *c, Route route, int M, int N, int K, const void *A, const void *B, void *C, int es,
                     size_t c_es, bool need_align, long pad) {
    const long lda = need_align ? round_up(K, pad) : K;
    const long rows = round_up((M + DevCtx::kMaxPanels - 1) / DevCtx::kMaxPanels, kPanelAlign);
    const int P = (int)((M + rows - 1) / rows);
    uint8_t *da = static_cast<uint8_t *>(stage_buf(c, 0, (size_t)lda * M * es));
    uint8_t *dc = static_cast<uint8_t *>(stage_buf(c, 2, (size_t)M * N * c_es));
    if (!da || !dc) return get_error();
    if (fault_injected("copy")) return X100_E_INJECTED;
    Operand b;
    if (!stage_in(c, 1, B, K, N, es, pad, need_align, b, c->up)) {
        cudaStreamSynchronize(c->up);
        return get_error();
    }
    const uint8_t *ha = static_cast<const uint8_t *>(A);
    uint8_t *hc = static_cast<uint8_t *>(C);
    int st = X100_OK;
    // fp32 on the tensor cores: B is split into its transposed tf32 high and
    // low parts once for all panels (slot 4), each panel's rows of A into
    // theirs (slot 5) as they arrive
    static const bool ffma = getenv("X100_GEMM_F32_FFMA") != nullptr;
    bool tf32 = route == ROUTE_F32_FAST && !ffma && tc_operands_ok(3, da, lda, b.dev, b.ld);
    const long ldt = (K + 3) & ~3L;
    float *bt = nullptr, *as = nullptr;
    if (tf32) {
        bt = static_cast<float *>(stage_buf(c, 4, (size_t)2 * N * ldt * 4));
        as = static_cast<float *>(stage_buf(c, 5, (size_t)2 * M * lda * 4));
        if (!bt || !as) st = get_error();
        cudaError_t e = cudaSuccess;
        if (!st) e = cudaEventRecord(c->ev[2 * DevCtx::kMaxPanels], c->up);
        if (!st && e == cudaSuccess) e = cudaStreamWaitEvent(c->stream, c->ev[2 * DevCtx::kMaxPanels], 0);
        if (!st && e != cudaSuccess) st = check_cuda(e, X100_E_COPY);
        if (!st)
            st = tf32_split_transpose(c, static_cast<const float *>(b.dev), b.ld, K, N, bt, bt + (size_t)N * ldt, ldt,
                                      c->stream);
    }
    for (int p = 0; p < P && st == X100_OK; ++p) {
        const long m0 = p * rows, mr = (M - m0 < rows) ? M - m0 : rows;
        const size_t c_off = (size_t)m0 * N * c_es, c_bytes = (size_t)mr * N * c_es;
        cudaError_t e = cudaMemcpy2DAsync(da + (size_t)m0 * lda * es, lda * es, ha + (size_t)m0 * K * es, (size_t)K * es,
                                          (size_t)K * es, mr, cudaMemcpyHostToDevice, c->up);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dc + c_off, hc + c_off, c_bytes, cudaMemcpyHostToDevice, c->up);
        if (e == cudaSuccess) e = cudaEventRecord(c->ev[p], c->up);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->stream, c->ev[p], 0);
        if (e != cudaSuccess) {
            st = check_cuda(e, X100_E_COPY);
            break;
        }
        if (tf32) {
            float *ahi = as + (size_t)m0 * lda, *alo = as + (size_t)M * lda + (size_t)m0 * lda;
            st = tf32_split(c, reinterpret_cast<const float *>(da + (size_t)m0 * lda * es), (long)mr * lda, ahi, alo,
                            c->stream);
            if (!st)
                st = launch_gemm_tf32x3(c, (int)mr, N, K, ahi, alo, lda, bt, bt + (size_t)N * ldt, ldt,
                                        reinterpret_cast<float *>(dc + c_off), N, c->stream);
            if (st == X100_E_UNSUPPORTED) {   // CTA pairs cannot run: the FFMA kernel from here on
                set_error(X100_OK);
                tf32 = false;
                st = X100_OK;
            }
        }
        if (!tf32 && !st)
            st = launch_route(c, route, (int)mr, N, K, da + (size_t)m0 * lda * es, lda, b.dev, b.ld, dc + c_off, N,
                              c->stream);
        if (st != X100_OK) break;
        e = cudaEventRecord(c->ev[DevCtx::kMaxPanels + p], c->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->down, c->ev[DevCtx::kMaxPanels + p], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(hc + c_off, dc + c_off, c_bytes, cudaMemcpyDeviceToHost, c->down);
        if (e != cudaSuccess) st = check_cuda(e, X100_E_COPY);
    }
    // every stream drains before the staging buffers can be reused
    const cudaError_t eu = cudaStreamSynchronize(c->up);
    const int sk = sync_and_status(c, c->stream);
    const cudaError_t ed = cudaStreamSynchronize(c->down);
    if (st == X100_OK && eu != cudaSuccess) st = check_cuda(eu, X100_E_COPY);
    if (st == X100_OK) st = sk;
    if (st == X100_OK && ed != cudaSuccess) st = check_cuda(ed, X100_E_COPY);
    return st;
}

// One synchronous host-API GEMM call.
void host_gemm(Route route, int M, int N, int K, const void *A, const void *B, void *C) {
    set_error(X100_OK);
    if (!dims_ok(M, N, K, A, B, C)) return;
    if (M == 0 || N == 0 || K == 0) return;
    DevCtx *c = ctx();
    if (!c) return;
    std::lock_guard<std::mutex> lk(c->mu);
    const bool is_i8 = route == ROUTE_TC_I8 || route == ROUTE_SIMT_I8;
    const bool is_f16 = route == ROUTE_F16_F32C || route == ROUTE_F16_F16C;
    const int es = is_i8 ? 1 : (is_f16 ? 2 : 4);
    const bool need_align = route == ROUTE_TC_I8 || route == ROUTE_F32_FAST || is_f16;
    const long pad = 16 / es;
    const size_t c_es = (route == ROUTE_F16_F16C) ? 2 : 4;
    const size_t moved = (size_t)M * K * es + (size_t)M * N * c_es;
    if (M >= 2 * kPanelAlign && moved >= kPanelMinBytes && !is_device_ptr(A) && !is_device_ptr(C)) {
        const int st = host_gemm_panels(c, route, M, N, K, A, B, C, es, c_es, need_align, pad);
        if (st != X100_OK) set_error(st);
        return;
    }
    Operand a, b;
    COperand co;
    if (!stage_in(c, 0, A, M, K, es, pad, need_align, a, c->stream) ||
        !stage_in(c, 1, B, K, N, es, pad, need_align, b, c->stream) || !stage_c(c, 2, C, (size_t)M * N * c_es, true, co))
        return;
    int st = launch_route(c, route, M, N, K, a.dev, a.ld, b.dev, b.ld, co.dev, N, c->stream);
    if (st != X100_OK) {
        cudaStreamSynchronize(c->stream);
        set_error(st);
        return;
    }
    st = finish_c(c, co);
    if (st != X100_OK) set_error(st);
}

// Asynchronous device-pointer GEMM: tensor cores when TMA can address the
// operands, CUDA cores otherwise.
int dev_gemm(Route route, int M, int N, int K, const void *A, long lda, const void *B, long ldb, void *C, long ldc,
             void *stream) {
    set_error(X100_OK);
    if (!dims_ok(M, N, K, A, B, C)) return X100_E_ARG;
    if (M == 0 || N == 0 || K == 0) return X100_OK;
    DevCtx *c = ctx();
    if (!c) return get_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st;
    switch (route) {
    case ROUTE_TC_I8:
        if (tc_operands_ok(0, A, lda, B, ldb))
            st = launch_gemm_tc(c, 0, M, N, K, A, lda, B, ldb, C, ldc, s);
        else
            st = launch_gemm_i8_simt(c, M, N, K, (const int8_t *)A, lda, (const int8_t *)B, ldb, (int32_t *)C, ldc, s);
        break;
    case ROUTE_SIMT_I8:
        st = launch_gemm_i8_simt(c, M, N, K, (const int8_t *)A, lda, (const int8_t *)B, ldb, (int32_t *)C, ldc, s);
        break;
    case ROUTE_F32_FAST:
        st = f32_fast(c, M, N, K, (const float *)A, lda, (const float *)B, ldb, (float *)C, ldc, s);
        break;
    case ROUTE_F32_REF:
        st = launch_gemm_f32_ref(c, M, N, K, (const float *)A, lda, (const float *)B, ldb, (float *)C, ldc, s);
        break;
    case ROUTE_F16_F32C:
    case ROUTE_F16_F16C: {
        const bool half_c = route == ROUTE_F16_F16C;
        if (tc_operands_ok(1, A, lda, B, ldb))
            st = launch_gemm_tc(c, half_c ? 2 : 1, M, N, K, A, lda, B, ldb, C, ldc, s);
        else
            st = launch_gemm_f16_simt(c, M, N, K, A, lda, B, ldb, C, ldc, half_c, s);
        break;
    }
    default: st = X100_E_ARG;
    }
    if (st != X100_OK) set_error(st);
    return st;
}

}  // namespace

extern "C" {

// ---- reference signatures (include/x100_gemm.h:50-61) -------------------------
void gemm_ref_f32(int M, int N, int K, const float *A, const float *B, float *C) {
    host_gemm(ROUTE_F32_REF, M, N, K, A, B, C);
}
void gemm_rvv_f32(int M, int N, int K, const float *A, const float *B, float *C) {
    host_gemm(ROUTE_F32_FAST, M, N, K, A, B, C);
}
void gemm_rvv_f16(int M, int N, int K, const _Float16 *A, const _Float16 *B, _Float16 *C) {
    host_gemm(ROUTE_F16_F16C, M, N, K, A, B, C);
}
void gemm_f16_f32acc(int M, int N, int K, const _Float16 *A, const _Float16 *B, float *C) {
    host_gemm(ROUTE_F16_F32C, M, N, K, A, B, C);
}
void gemm_ref_i8(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C) {
    host_gemm(ROUTE_SIMT_I8, M, N, K, A, B, C);
}
void gemm_ime_i8(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C) {
    host_gemm(ROUTE_TC_I8, M, N, K, A, B, C);
}

// ---- device-pointer variants ---------------------------------------------------------
int gemm_ime_i8_dev(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, void *stream) {
    return dev_gemm(ROUTE_TC_I8, M, N, K, A, K, B, N, C, N, stream);
}
int gemm_ref_i8_dev(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, void *stream) {
    return dev_gemm(ROUTE_SIMT_I8, M, N, K, A, K, B, N, C, N, stream);
}
int gemm_f16_f32acc_dev(int M, int N, int K, const void *A, const void *B, float *C, void *stream) {
    return dev_gemm(ROUTE_F16_F32C, M, N, K, A, K, B, N, C, N, stream);
}
int gemm_f16_dev(int M, int N, int K, const void *A, const void *B, void *C, void *stream) {
    return dev_gemm(ROUTE_F16_F16C, M, N, K, A, K, B, N, C, N, stream);
}
int gemm_f32_dev(int M, int N, int K, const float *A, const float *B, float *C, void *stream) {
    return dev_gemm(ROUTE_F32_FAST, M, N, K, A, K, B, N, C, N, stream);
}
int gemm_ref_f32_dev(int M, int N, int K, const float *A, const float *B, float *C, void *stream) {
    return dev_gemm(ROUTE_F32_REF, M, N, K, A, K, B, N, C, N, stream);
}
// Strided device variant: explicit leading dimensions (elements).
int gemm_ime_i8_dev_ld(int M, int N, int K, const int8_t *A, long lda, const int8_t *B, long ldb, int32_t *C,
                       long ldc, void *stream) {
    return dev_gemm(ROUTE_TC_I8, M, N, K, A, lda, B, ldb, C, ldc, stream);
}

// ---- packed-operand driver (src/gemm_ime2_i8.c:40-147) --------------------------
static int ime2_check(int Mt, int Nt, int Kt, const void *a, const void *b) {
    if (Mt <= 0 || Nt <= 0 || Kt <= 0 || Mt % 8 || Nt % 64 || Kt % 16 || !a || !b) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    return X100_OK;
}

// Layout conversions run on the host: they only move bytes (the reference's
// packers are plain host loops too, src/gemm_ime2_i8.c:40-56).
void gemm_ime2_pack_a(int Mt, int Kt, const int8_t *A, int8_t *pa) {
    set_error(X100_OK);
    if (Mt % 8 || Kt % 16 || Mt < 0 || Kt < 0 || !A || !pa) {
        set_error(X100_E_ARG);
        return;
    }
    const int Mb = Mt / 8, Kb = Kt / 16;
    for (int mb = 0; mb < Mb; ++mb)
        for (int kb = 0; kb < Kb; ++kb) {
            int8_t *d = pa + ((size_t)mb * Kb + kb) * 128;
            for (int r = 0; r < 8; ++r) memcpy(d + r * 16, A + (size_t)(mb * 8 + r) * Kt + kb * 16, 16);
        }
}
void gemm_ime2_pack_b(int Kt, int Nt, const int8_t *B, int8_t *pb) {
    set_error(X100_OK);
    if (Nt % 64 || Kt % 16 || Nt < 0 || Kt < 0 || !B || !pb) {
        set_error(X100_E_ARG);
        return;
    }
    const int Kb = Kt / 16, Ng = Nt / 64;
    for (int ng = 0; ng < Ng; ++ng)
        for (int kb = 0; kb < Kb; ++kb)
            for (int g = 0; g < 8; ++g) {
                int8_t *d = pb + (((size_t)ng * Kb + kb) * 8 + g) * 128;
                const int nb = ng * 8 + g;
                for (int nin = 0; nin < 8; ++nin)
                    for (int kin = 0; kin < 16; ++kin) d[nin * 16 + kin] = B[(size_t)(kb * 16 + kin) * Nt + nb * 8 + nin];
            }
}

void gemm_ime2_i8_st(int Mt, int Nt, int Kt, const int8_t *pa, const int8_t *pb, int32_t *C) {
    gemm_ime2_i8_mt(Mt, Nt, Kt, pa, pb, C, 1);
}

void gemm_ime2_i8_mt(int Mt, int Nt, int Kt, const int8_t *pa, const int8_t *pb, int32_t *C, int nthreads) {
    (void)nthreads;
    set_error(X100_OK);
    if (ime2_check(Mt, Nt, Kt, pa, pb) || !C) {
        set_error(X100_E_ARG);
        return;
    }
    DevCtx *c = ctx();
    if (!c) return;
    std::lock_guard<std::mutex> lk(c->mu);
    const size_t na = (size_t)Mt * Kt, nb = (size_t)Kt * Nt, nc = (size_t)Mt * Nt * 4;
    Operand a, b;
    COperand co;
    // packed operands (slots 0, 1), row-major operands (slot 3 holds both), C (slot 2)
    if (!stage_in(c, 0, pa, 1, (long)na, 1, 16, false, a, c->stream) ||
        !stage_in(c, 1, pb, 1, (long)nb, 1, 16, false, b, c->stream) ||
        !stage_c(c, 2, C, nc, false, co))
        return;
    int8_t *rm = static_cast<int8_t *>(stage_buf(c, 3, na + nb));
    if (!rm) return;
    int st = launch_ime2_unpack(c, Mt, Nt, Kt, (const int8_t *)a.dev, (const int8_t *)b.dev, rm, rm + na, c->stream);
    if (st == X100_OK) st = check_cuda(cudaMemsetAsync(co.dev, 0, nc, c->stream), X100_E_LAUNCH);
    if (st == X100_OK) st = launch_gemm_tc(c, 0, Mt, Nt, Kt, rm, Kt, rm + na, Nt, co.dev, Nt, c->stream);
    if (st != X100_OK) {
        cudaStreamSynchronize(c->stream);
        set_error(st);
        return;
    }
    st = finish_c(c, co);
    if (st != X100_OK) set_error(st);
}

}  // extern "C"
