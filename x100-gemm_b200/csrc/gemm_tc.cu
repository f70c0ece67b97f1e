// gemm_tc.cu -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M x N] += A[M x K] * B[K x N]   (row-major; A is K-major, B is N-major)
//
// kind::i8 (int8 x int8 -> int32, exact) replaces the reference's
// gemm_ime_i8 / IME-2 ukernel_8x64 (src/gemm_ime_i8.c:60-89,
// src/gemm_ime2_i8.c:60-147); kind::f16 (fp16 x fp16 -> fp32 accumulate)
// replaces gemm_rvv_f16 (src/gemm_rvv_f16.c:15-57).
//
// Structure (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0   TMA producer: per 128-byte K slab, one A box (128 rows x 128 B)
//            and 256/atom B boxes (K rows x 128 B of N), 128-byte swizzle,
//            into a 4-stage shared-memory ring guarded by mbarriers.
//   warp 1   MMA issuer: one thread issues 4 tcgen05.mma (M=128, N=256,
//            K = 32 bytes) per slab into a TMEM accumulator; two
//            accumulators (2 x 256 columns = all 512 TMEM columns) let the
//            epilogue of tile i overlap the main loop of tile i+1.
//   warps 2-5 epilogue: tcgen05.ld 32 lanes x 32 columns, transpose through
//            a padded shared buffer, then coalesced C read-add-write (beta=1).
// Every mbarrier wait is bounded (see ptx.cuh); on a timeout the kernel
// records X100_E_TIMEOUT in the status word, drains its in-flight TMA copies
// and MMAs, frees its TMEM and returns.
#include <cuda_fp16.h>

#include "gemm_kernels.h"
#include "ptx.cuh"

namespace x100 {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * 128;   // one stage of A: 128 rows x 128 bytes of K
constexpr int B_BYTES = BN * 128;   // one stage of B: 128 bytes of K (rows) x 256 columns
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_LD = 33;          // padded row (words) of the transpose buffer
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_LD * 4;
constexpr int BAR_OFF = STAGES * STAGE_BYTES + EPI_BYTES;
constexpr int NBARS = 2 * STAGES + 2 + 2 + 1;
constexpr int SMEM_BYTES = BAR_OFF + NBARS * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr int GROUP_M = 16;         // tile raster: 16 M-tiles share each B panel
constexpr unsigned long long kDrainNs = 100000000ull;

template <int KIND> struct Traits;
template <> struct Traits<0> { static constexpr int ES = 1; using CT = int32_t; };
template <> struct Traits<1> { static constexpr int ES = 2; using CT = float; };
template <> struct Traits<2> { static constexpr int ES = 2; using CT = __half; };

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int &mt, int &nt) {
    const int group = GROUP_M * num_n;
    const int g = tile / group;
    const int first_m = g * GROUP_M;
    const int gm = min(num_m - first_m, GROUP_M);
    const int r = tile - g * group;
    mt = first_m + r % gm;
    nt = r / gm;
}

// C element update c + acc for each output type (int32 adds wrap modulo 2^32
// like the CPU reference; fp16 C is widened, added in fp32, rounded once).
__device__ __forceinline__ int32_t epi_add(int32_t c, uint32_t v) {
    return static_cast<int32_t>(static_cast<uint32_t>(c) + v);
}
__device__ __forceinline__ float epi_add(float c, uint32_t v) { return c + __uint_as_float(v); }
__device__ __forceinline__ __half epi_add(__half c, uint32_t v) {
    return __float2half_rn(__half2float(c) + __uint_as_float(v));
}

// Read-add-write of `rows` (<= 32) rows of one 32-column chunk; lane owns a
// column, so every row access is one coalesced 32-element segment.  Loads
// are batched ahead of the stores to keep many requests in flight.
template <typename CT>
__device__ __forceinline__ void epi_rows(CT *cp, long ldc, const uint32_t *buf, int lane, int rows) {
    if (rows == 32) {
#pragma unroll
        for (int i0 = 0; i0 < 32; i0 += 16) {
            CT v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = cp[static_cast<long>(i0 + j) * ldc];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                cp[static_cast<long>(i0 + j) * ldc] = epi_add(v[j], buf[(i0 + j) * EPI_LD + lane]);
        }
    } else {
        for (int i = 0; i < rows; ++i)
            cp[static_cast<long>(i) * ldc] = epi_add(cp[static_cast<long>(i) * ldc], buf[i * EPI_LD + lane]);
    }
}

template <int KIND>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   typename Traits<KIND>::CT *__restrict__ C, int M, int N, int K, long ldc, int *status) {
    using CT = typename Traits<KIND>::CT;
    constexpr int ES = Traits<KIND>::ES;
    constexpr int BK = 128 / ES;          // K elements per stage
    constexpr int UK = 32 / ES;           // K elements per MMA
    constexpr int KSTEPS = BK / UK;       // MMAs per stage (4)
    constexpr int ATOM_N = 128 / ES;      // N elements per 128-byte swizzle atom
    constexpr int NBOX = BN / ATOM_N;     // B boxes per stage
    constexpr int BOX_B_BYTES = BK * 128; // one B box: BK rows x 128 bytes
    constexpr uint32_t IDESC = (KIND == 0) ? idesc_make(2, 1, 1, BM, BN) : idesc_make(1, 0, 1, BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    uint32_t *epi = reinterpret_cast<uint32_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BAR_OFF);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int total = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t stage = 0, phase = 0;
            uint32_t issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                int mt, nt;
                tile_coords(tile, num_m, num_n, mt, nt);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, mt * BM, &full[stage]);
#pragma unroll
                    for (int j = 0; j < NBOX; ++j)
                        tma_load_2d(sB + stage * B_BYTES + j * BOX_B_BYTES, &tmB, nt * BN + j * ATOM_N, kb * BK,
                                    &full[stage]);
                    issued[stage]++;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (ok) {
                // wait until the MMA warp has released every stage it will use
                for (int i = 0; i < STAGES; ++i) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status)) break;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            } else {
                // aborting: wait (bounded) for the copies already in flight
                for (int s = 0; s < STAGES; ++s)
                    if (issued[s]) mbar_wait_drain(&full[s], (issued[s] - 1u) & 1u, kDrainNs);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int k = 0; k < KSTEPS; ++k) {
                        const uint64_t adesc = smem_desc_sw128(a0 + k * 32, 16, 1024);
                        const uint64_t bdesc = smem_desc_sw128(b0 + k * UK * 128, BOX_B_BYTES, 1024);
                        if (KIND == 0)
                            umma_i8(d_tmem, adesc, bdesc, IDESC, (kb | k) ? 1u : 0u);
                        else
                            umma_f16(d_tmem, adesc, bdesc, IDESC, (kb | k) ? 1u : 0u);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            // all MMAs issued by this thread complete before TMEM is freed
            umma_commit(drain);
            mbar_wait_drain(drain, 0, kDrainNs);
        }
    } else {
        // ---------------- epilogue ----------------
        const int q = warp & 3;   // TMEM lane quadrant this warp may access
        uint32_t *buf = epi + (warp - 2) * 32 * EPI_LD;
        uint32_t acc = 0, acc_phase = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            int mt, nt;
            tile_coords(tile, num_m, num_n, mt, nt);
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, status)) break;
            tc_fence_after();
            const int row0 = mt * BM + q * 32;
            const int n0 = nt * BN;
            const int nchunks = min(BN / 32, (N - n0 + 31) / 32);
            for (int c = 0; c < nchunks; ++c) {
                uint32_t r[32];
                tmem_ld32(tmem_base + acc * BN + c * 32 + (static_cast<uint32_t>(q * 32) << 16), r);
                tmem_wait_ld();
                if (c == nchunks - 1) {
                    // accumulator fully read: hand it back to the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) buf[lane * EPI_LD + j] = r[j];
                __syncwarp();
                const int col = n0 + c * 32 + lane;
                if (row0 < M && col < N)
                    epi_rows<CT>(C + static_cast<long>(row0) * ldc + col, ldc, buf, lane, min(32, M - row0));
                __syncwarp();
            }
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int KIND>
static int launch_kind(DevCtx *c, int M, int N, int K, const void *A, long lda, const void *B, long ldb, void *C,
                       long ldc, cudaStream_t s) {
    constexpr int ES = Traits<KIND>::ES;
    constexpr int BK = 128 / ES;
    constexpr int ATOM_N = 128 / ES;
    const CUtensorMapDataType dt = (KIND == 0) ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, dt, (uint64_t)K, (uint64_t)M, (uint64_t)lda * ES, BK, BM) ||
        !make_tmap_2d(&tb, B, dt, (uint64_t)N, (uint64_t)K, (uint64_t)ldb * ES, ATOM_N, BK)) {
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    static bool attr_set[64] = {};
    if (!attr_set[c->device]) {
        if (cudaFuncSetAttribute(gemm_tc_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
        attr_set[c->device] = true;
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < c->sm_count ? tiles : c->sm_count;
    gemm_tc_kernel<KIND><<<grid, THREADS, SMEM_BYTES, s>>>(ta, tb, reinterpret_cast<typename Traits<KIND>::CT *>(C),
                                                          M, N, K, ldc, c->d_status);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

}  // namespace tc

bool tc_operands_ok(int kind, const void *A, long lda, const void *B, long ldb) {
    const int es = kind == 0 ? 1 : 2;
    return (reinterpret_cast<uintptr_t>(A) % 16 == 0) && (reinterpret_cast<uintptr_t>(B) % 16 == 0) &&
           ((lda * es) % 16 == 0) && ((ldb * es) % 16 == 0);
}

int launch_gemm_tc(DevCtx *c, int kind, int M, int N, int K, const void *A, long lda, const void *B, long ldb,
                   void *C, long ldc, cudaStream_t s) {
    if (c->cc_major != 10) {
        set_error(X100_E_ARCH);
        return X100_E_ARCH;
    }
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    switch (kind) {
    case 0: return tc::launch_kind<0>(c, M, N, K, A, lda, B, ldb, C, ldc, s);
    case 1: return tc::launch_kind<1>(c, M, N, K, A, lda, B, ldb, C, ldc, s);
    case 2: return tc::launch_kind<2>(c, M, N, K, A, lda, B, ldb, C, ldc, s);
    default: set_error(X100_E_ARG); return X100_E_ARG;
    }
}

}  // namespace x100
