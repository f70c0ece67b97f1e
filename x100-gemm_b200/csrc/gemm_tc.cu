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

#include <cstdlib>

#include "gemm_kernels.h"
#include "ptx.cuh"

namespace x100 {
bool pdl_enabled();   // qgemv.cu: false when X100_NO_PDL is set
}

namespace x100 {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;         // two per TMEM lane quadrant, each takes half the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * 128;   // one stage of A: 128 rows x 128 bytes of K
constexpr int B_BYTES = BN * 128;   // one stage of B: 128 bytes of K (rows) x 256 columns
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_LD = 33;          // padded row (words) of an epilogue warp's transpose buffer
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_LD * 4;
constexpr int BAR_OFF = STAGES * STAGE_BYTES + EPI_BYTES;   // stages, then the transpose buffers
constexpr int NBARS = 2 * STAGES + 2 + 2 + 1;
constexpr int SMEM_BYTES = BAR_OFF + NBARS * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr int GROUP_M = 16;         // tile raster: 16 M-tiles share each B panel
constexpr unsigned long long kDrainNs = 100000000ull;

template <int KIND> struct Traits;
template <> struct Traits<0> { static constexpr int ES = 1; using CT = int32_t; };
template <> struct Traits<1> { static constexpr int ES = 2; using CT = float; };
template <> struct Traits<2> { static constexpr int ES = 2; using CT = __half; };
// kind 3: fp32 x fp32 -> fp32 as three kind::tf32 products (A_hi.B_hi +
// A_hi.B_lo + A_lo.B_hi, X_hi = X rounded to tf32, X_lo = X - X_hi), 2-SM
// kernel only.  B and B_lo come transposed (N x K, both
// operands K-major): kind::tf32 with an N-major B produced zeros here.
template <> struct Traits<3> { static constexpr int ES = 4; using CT = float; };

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int &mt, int &nt) {
    const int group = GROUP_M * num_n;
    const int g = tile / group;
    const int first_m = g * GROUP_M;
    const int gm = min(num_m - first_m, GROUP_M);
    const int r = tile - g * group;
    mt = first_m + r % gm;
    nt = r / gm;
}

// Work list of one CTA pair of the 2-SM kernel.  Whole output tiles come
// first, tile = pair + j * npairs, for the full waves; with stream-K on, the
// tiles of the last, partial wave are cut along K instead: their
// (tile, k-block) units are split into `spairs` contiguous runs of at least
// kMinSkBlocks k-blocks, one run per pair, so every pair ends at about the
// same time.  A run can cover the end of one tile and the start of the next;
// each piece is accumulated in TMEM from zero and added to C by the TMA
// reduce-add epilogue, whose element-wise integer adds make the result
// independent of the order in which the pieces land.  Every role of a pair
// (TMA producer, MMA issuer, epilogue warps) walks the same list.
constexpr int kMinSkBlocks = 8;

__host__ __device__ inline int sk_pairs(int total, int num_kb, int npairs) {
    const int rem = total % npairs;
    const long units = (long)rem * num_kb;
    const long sp = units / kMinSkBlocks < npairs ? units / kMinSkBlocks : npairs;
    return (rem > 0 && sp > rem) ? (int)sp : 0;   // no gain unless more pairs than tiles share the tail
}

// kp < num_kb (fp32 and fp16 -> fp32 kinds): every whole tile is further cut into
// consecutive K-pieces of kp k-blocks, taken in order by the same pair, each
// accumulated from zero and added into C -- so no accumulator sums more than
// kp k-blocks (the tensor core's fp32 accumulation loses low bits at every
// step, an error that grows with the steps of one accumulator).
struct PairSched {
    int npairs, pair, num_kb, dp_tiles, j = 0, kp, piece = 0;
    long it = 0, end = 0;
    __device__ PairSched(int total, int num_kb_, int npairs_, int pair_, bool sk, int kp_ = 1 << 30)
        : npairs(npairs_), pair(pair_), num_kb(num_kb_), dp_tiles(total), kp(kp_ < num_kb_ ? kp_ : num_kb_) {
        const int sp = sk ? sk_pairs(total, num_kb, npairs) : 0;
        if (sp > 0) {
            const int rem = total % npairs;
            const long units = (long)rem * num_kb;
            dp_tiles = total - rem;
            if (pair < sp) {
                it = (long)dp_tiles * num_kb + units * pair / sp;
                end = (long)dp_tiles * num_kb + units * (pair + 1) / sp;
            }
        }
    }
    // next piece: output tile and its k-blocks [kb0, kb1)
    __device__ bool next(int &tile, int &kb0, int &kb1) {
        const int t = pair + j * npairs;
        if (t < dp_tiles) {
            tile = t;
            kb0 = piece * kp;
            kb1 = kb0 + kp < num_kb ? kb0 + kp : num_kb;
            if (kb1 >= num_kb) {
                ++j;
                piece = 0;
            } else {
                ++piece;
            }
            return true;
        }
        if (it < end) {
            tile = (int)(it / num_kb);
            kb0 = (int)(it - (long)tile * num_kb);
            const long left = end - it;
            kb1 = left < num_kb - kb0 ? kb0 + (int)left : num_kb;
            it += kb1 - kb0;
            return true;
        }
        return false;
    }
};

// C element update c + acc for each output type (int32 adds wrap modulo 2^32
// like the CPU reference; fp16 C is widened, added in fp32, rounded once).
__device__ __forceinline__ int32_t epi_add(int32_t c, uint32_t v) {
    return static_cast<int32_t>(static_cast<uint32_t>(c) + v);
}
__device__ __forceinline__ float epi_add(float c, uint32_t v) { return c + __uint_as_float(v); }
__device__ __forceinline__ __half epi_add(__half c, uint32_t v) {
    return __float2half_rn(__half2float(c) + __uint_as_float(v));
}

// ---- epilogue: C += accumulator ------------------------------------------------------
// Epilogue warp w (w >= 2) may read TMEM lanes 32 * (w % 4) .. +31, i.e. rows
// 32q .. 32q+31 of the CTA's accumulator (q = w % 4); the two warps of a
// quadrant split the 32-column chunks.  A chunk arrives from tcgen05.ld with
// one row per thread; it is transposed through a padded per-warp buffer so
// that each C access of the warp is one full 128-byte row segment (lane =
// column; whole sectors, coalesced).  The C rows of a chunk are read ahead:
// the first chunk before the accumulator is ready, each next chunk while the
// current one is added and stored.
// One accumulator (tile) of this warp: rows row_base + 32q .. +31, column
// chunks [c0, c1) from n0.  Waits for the accumulator (tfull), releases it
// (arrive on the barrier at release_addr, a shared::cluster address) once
// read.  Returns false on a timeout.
template <typename CT>
__device__ __forceinline__ bool epi_tile(uint32_t tmem_acc, int q, int lane, int c0, int c1, CT *__restrict__ C,
                                         long ldc, int M, int N, int row_base, int n0, uint64_t *tfull,
                                         uint32_t parity, uint32_t release_addr, uint32_t *buf,
                                         volatile int *abort_flag, int *status) {
    const int r0 = row_base + q * 32;
    const int nrows = max(0, min(32, M - r0));
    auto load = [&](int c, CT (&v)[32]) {
        const int col = n0 + c * 32 + lane;
        if (c < c1 && col < N) {
            const CT *p = C + static_cast<long>(r0) * ldc + col;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < nrows) v[i] = __ldcs(p + static_cast<long>(i) * ldc);
        }
    };
    CT cur[32];
    load(c0, cur);
    if (!mbar_wait(tfull, parity, abort_flag, status)) return false;
    tc_fence_after();
    if (c0 >= c1) {   // nothing of this tile for this warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(release_addr);
        return true;
    }
    for (int c = c0; c < c1; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_acc + c * 32 + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_wait_ld();
        if (c == c1 - 1) {   // accumulator fully read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(release_addr);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) buf[lane * EPI_LD + j] = r[j];
        __syncwarp();
        CT nxt[32];
        load(c + 1, nxt);
        const int col = n0 + c * 32 + lane;
        if (col < N) {
            CT *p = C + static_cast<long>(r0) * ldc + col;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < nrows) __stcs(p + static_cast<long>(i) * ldc, epi_add(cur[i], buf[i * EPI_LD + lane]));
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; ++i) cur[i] = nxt[i];
    }
    return true;
}

// The same for 32-bit C whose tensor map allows TMA: the chunk goes from
// TMEM through a 4 KB per-warp buffer (128-byte swizzle: row r's 16-byte
// piece i sits at position i ^ (r % 8), so the 8 lanes of a quarter-warp
// write 8 distinct bank groups) and is added into C by one TMA reduce-add,
// so C never passes through the SM (the L2 reads, adds and writes it).
__device__ __forceinline__ bool epi_tile_tma(uint32_t tmem_acc, int q, int lane, int c0, int c1,
                                             const CUtensorMap *tmC, int row_base, int n0, uint64_t *tfull,
                                             uint32_t parity, uint32_t release_addr, uint8_t *buf,
                                             volatile int *abort_flag, int *status) {
    if (!mbar_wait(tfull, parity, abort_flag, status)) return false;
    tc_fence_after();
    if (c0 >= c1) {   // nothing of this tile for this warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(release_addr);
        return true;
    }
    for (int c = c0; c < c1; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_acc + c * 32 + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_wait_ld();
        if (c == c1 - 1) {   // accumulator fully read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(release_addr);
        }
        if (lane == 0) bulk_wait_read_all();   // the previous chunk's reduce has read the buffer
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4 *>(buf + lane * 128 + ((i ^ (lane & 7)) << 4)) =
                make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_reduce_add_2d(tmC, n0 + c * 32, row_base + q * 32, buf);
            bulk_commit();
        }
    }
    return true;
}

// TE: C += accumulator by TMA reduce-add (32-bit C with a TMA-compatible layout)
template <int KIND, bool TE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, typename Traits<KIND>::CT *__restrict__ C, int M, int N,
                   int K, long ldc, int *status) {
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
        const int h = (warp - 2) >> 2;
        uint32_t *buf = reinterpret_cast<uint32_t *>(smem + STAGES * STAGE_BYTES) + (warp - 2) * 32 * EPI_LD;
        uint8_t *tbuf = smem + STAGES * STAGE_BYTES + (warp - 2) * 4096;   // 1024-aligned (TE)
        const uint32_t rel[2] = {smem_u32(&tempty[0]), smem_u32(&tempty[1])};
        uint32_t acc = 0, acc_phase = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            int mt, nt;
            tile_coords(tile, num_m, num_n, mt, nt);
            const int n0 = nt * BN;
            const int nchunks = min(BN / 32, (N - n0 + 31) / 32);
            const int c0 = min(h * (BN / 64), nchunks), c1 = min((h + 1) * (BN / 64), nchunks);
            bool ok;
            if constexpr (TE)
                ok = epi_tile_tma(tmem_base + acc * BN, q, lane, c0, c1, &tmC, mt * BM, n0, &tfull[acc], acc_phase,
                                  rel[acc], tbuf, abort_flag, status);
            else
                ok = epi_tile<CT>(tmem_base + acc * BN, q, lane, c0, c1, C, ldc, M, N, mt * BM, n0, &tfull[acc],
                                  acc_phase, rel[acc], buf, abort_flag, status);
            if (!ok) break;
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    if (TE && warp >= 2 && lane == 0) bulk_wait_all();   // this warp's reduce-adds into C are done
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- 2-SM version: one CTA pair (cluster of 2) per 256 x 256 output tile ----------------
// Each CTA stages its 128 rows of A and its 128 columns of B (32 KB per
// 128-byte K slab, six stages); the pair leader (CTA rank 0) issues
// tcgen05.mma.cta_group::2 with M = N = 256, whose accumulator rows 0-127
// live in the leader's TMEM and rows 128-255 in the peer's.  Per output
// element this halves the bytes each SM pulls from L2 compared with the
// 128 x 256 single-CTA tile.  Both CTAs' copies complete on the leader's
// `full` barrier (the leader announces both halves); the leader's commits
// arrive on the `empty` / `tfull` barriers of both CTAs; both epilogues
// release an accumulator on the leader's `tempty` barrier.
constexpr int P_STAGES = 6;
constexpr int P_ROWS = 128;                       // A rows (and C rows) per CTA
constexpr int P_COLS = 128;                       // B columns per CTA
constexpr int P_A_BYTES = P_ROWS * 128;
constexpr int P_B_BYTES = P_COLS * 128;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_BAR_OFF = P_STAGES * P_STAGE_BYTES + EPI_BYTES;
constexpr int P_NBARS = 2 * P_STAGES + 2 + 2 + 1;
constexpr int P_SMEM_BYTES = P_BAR_OFF + P_NBARS * 8 + 16 + 1024;

template <int KIND, bool TE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmA2,
                    const __grid_constant__ CUtensorMap tmB2, typename Traits<KIND>::CT *__restrict__ C, int M,
                    int N, int K, long ldc, int sk, int kp, int *status) {
    using CT = typename Traits<KIND>::CT;
    constexpr int ES = Traits<KIND>::ES;
    constexpr int BK = 128 / ES;          // K elements per stage
    constexpr int UK = 32 / ES;           // K elements per MMA
    constexpr int KSTEPS = BK / UK;       // MMAs per stage (4)
    constexpr int ATOM_N = 128 / ES;      // N elements per 128-byte swizzle atom
    constexpr int NBOX = P_COLS / ATOM_N; // B boxes per stage per CTA
    constexpr int BOX_B_BYTES = BK * 128;
    constexpr int TM = 2 * P_ROWS, TN = 2 * P_COLS;   // output tile of the pair
    constexpr uint32_t IDESC = (KIND == 0)   ? idesc_make(2, 1, 1, TM, TN)
                               : (KIND == 3) ? idesc_make(1, 2, 0, TM, TN)
                                             : idesc_make(1, 0, 1, TM, TN);
    // kind 3 stages hold the low parts too: [A | A_lo] and [B | B_lo], in
    // half as many stages of the same total size
    constexpr int NOPS = (KIND == 3) ? 2 : 1;
    constexpr int PA = NOPS * P_A_BYTES, PB = NOPS * P_B_BYTES, PSTAGES = P_STAGES / NOPS;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + PSTAGES * PA;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_BAR_OFF);
    uint64_t *full = bars;
    uint64_t *empty = bars + P_STAGES;
    uint64_t *tfull = bars + 2 * P_STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + P_NBARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();                  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic dependent launch, the CTA may start while the
    // previous kernel of the stream runs: the setup above overlaps its tail,
    // and nothing touches A, B or C before it has completed.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int num_m = (M + TM - 1) / TM;
    const int num_n = (N + TN - 1) / TN;
    const int total = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            uint32_t stage = 0, phase = 0;
            uint32_t issued[P_STAGES];
            for (int s = 0; s < P_STAGES; ++s) issued[s] = 0;
            uint32_t full_l[P_STAGES];
            for (int s = 0; s < P_STAGES; ++s) full_l[s] = mapa_shared(&full[s], 0);
            bool ok = true;
            PairSched sched(total, num_kb, npairs, pair, sk != 0, kp);
            int tile, kb0, kb1;
            while (ok && sched.next(tile, kb0, kb1)) {
                int mt, nt;
                tile_coords(tile, num_m, num_n, mt, nt);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (PA + PB));
                    tma_load_2d_pair(sA + stage * PA, &tmA, kb * BK, mt * TM + (int)rank * P_ROWS, full_l[stage]);
                    if constexpr (KIND == 3)
                        tma_load_2d_pair(sA + stage * PA + P_A_BYTES, &tmA2, kb * BK, mt * TM + (int)rank * P_ROWS,
                                         full_l[stage]);
                    if constexpr (KIND == 3) {   // B^T and B_lo^T: K-major, one box each
                        tma_load_2d_pair(sB + stage * PB, &tmB, kb * BK, nt * TN + (int)rank * P_COLS, full_l[stage]);
                        tma_load_2d_pair(sB + stage * PB + P_B_BYTES, &tmB2, kb * BK, nt * TN + (int)rank * P_COLS,
                                         full_l[stage]);
                    } else {
#pragma unroll
                        for (int j = 0; j < NBOX; ++j)
                            tma_load_2d_pair(sB + stage * PB + j * BOX_B_BYTES, &tmB,
                                             nt * TN + (int)rank * P_COLS + j * ATOM_N, kb * BK, full_l[stage]);
                    }
                    issued[stage]++;
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (ok) {
                // wait until the leader's MMAs have released every stage
                for (int i = 0; i < PSTAGES; ++i) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status)) break;
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            } else if (leader) {
                // aborting: wait (bounded) for the copies of both CTAs announced so far
                for (int s = 0; s < PSTAGES; ++s)
                    if (issued[s]) mbar_wait_drain(&full[s], (issued[s] - 1u) & 1u, kDrainNs);
            } else {
                // aborting: this CTA's copies complete on the leader's barrier; give them
                // time to land before the shared memory is released
                const unsigned long long t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (pair leader) ----------------
            uint32_t empty_p[P_STAGES], tfull_p[2];
            for (int s = 0; s < P_STAGES; ++s) empty_p[s] = mapa_shared(&empty[s], 1);
            for (int b = 0; b < 2; ++b) tfull_p[b] = mapa_shared(&tfull[b], 1);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            PairSched sched(total, num_kb, npairs, pair, sk != 0, kp);
            int tile, kb0, kb1;
            while (ok && sched.next(tile, kb0, kb1)) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * TN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * PA);
                    const uint32_t b0 = smem_u32(sB + stage * PB);
#pragma unroll
                    for (int k = 0; k < KSTEPS; ++k) {
                        const uint64_t adesc = smem_desc_sw128(a0 + k * 32, 16, 1024);
                        const uint64_t bdesc = smem_desc_sw128(b0 + k * UK * 128, BOX_B_BYTES, 1024);
                        const uint32_t accum = (kb != kb0 || k) ? 1u : 0u;
                        if constexpr (KIND == 0) {
                            umma_i8_pair(d_tmem, adesc, bdesc, IDESC, accum);
                        } else if constexpr (KIND == 3) {   // all four operands K-major
                            const uint64_t a2desc = smem_desc_sw128(a0 + P_A_BYTES + k * 32, 16, 1024);
                            const uint64_t bkdesc = smem_desc_sw128(b0 + k * 32, 16, 1024);
                            const uint64_t b2desc = smem_desc_sw128(b0 + P_B_BYTES + k * 32, 16, 1024);
                            umma_tf32_pair(d_tmem, adesc, bkdesc, IDESC, accum);
                            umma_tf32_pair(d_tmem, adesc, b2desc, IDESC, 1u);
                            umma_tf32_pair(d_tmem, a2desc, bkdesc, IDESC, 1u);
                        } else {
                            umma_f16_pair(d_tmem, adesc, bdesc, IDESC, accum);
                        }
                    }
                    umma_commit_pair(smem_u32(&empty[stage]));
                    umma_commit_pair(empty_p[stage]);
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(smem_u32(&tfull[acc]));
                umma_commit_pair(tfull_p[acc]);
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            // all MMAs issued by this thread complete before TMEM is freed
            umma_commit_pair(smem_u32(drain));
            mbar_wait_drain(drain, 0, kDrainNs);
        }
    } else {
        // ---------------- epilogue (both CTAs) ----------------
        const int q = warp & 3;   // TMEM lane quadrant this warp may access
        const int h = (warp - 2) >> 2;
        uint32_t *buf = reinterpret_cast<uint32_t *>(smem + PSTAGES * (PA + PB)) + (warp - 2) * 32 * EPI_LD;
        uint8_t *tbuf = smem + PSTAGES * (PA + PB) + (warp - 2) * 4096;   // 1024-aligned (TE)
        const uint32_t rel[2] = {mapa_shared(&tempty[0], 0), mapa_shared(&tempty[1], 0)};
        uint32_t acc = 0, acc_phase = 0;
        PairSched sched(total, num_kb, npairs, pair, sk != 0, kp);
        int tile, kb0, kb1;
        while (sched.next(tile, kb0, kb1)) {
            int mt, nt;
            tile_coords(tile, num_m, num_n, mt, nt);
            const int n0 = nt * TN;
            const int nchunks = min(TN / 32, (N - n0 + 31) / 32);
            const int c0 = min(h * (TN / 64), nchunks), c1 = min((h + 1) * (TN / 64), nchunks);
            bool ok;
            if constexpr (TE)
                ok = epi_tile_tma(tmem_base + acc * TN, q, lane, c0, c1, &tmC, mt * TM + (int)rank * P_ROWS, n0,
                                  &tfull[acc], acc_phase, rel[acc], tbuf, abort_flag, status);
            else
                ok = epi_tile<CT>(tmem_base + acc * TN, q, lane, c0, c1, C, ldc, M, N, mt * TM + (int)rank * P_ROWS,
                                  n0, &tfull[acc], acc_phase, rel[acc], buf, abort_flag, status);
            if (!ok) break;
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    if (TE && warp >= 2 && lane == 0) bulk_wait_all();   // this warp's reduce-adds into C are done
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();                  // no arrival into either CTA is still pending
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
    cluster_sync_all();
}

template <int KIND, bool TE>
static int launch_te(DevCtx *c, int M, int N, int K, const CUtensorMap &ta, const CUtensorMap &tb,
                     const CUtensorMap &tc_, const CUtensorMap &ta2, const CUtensorMap &tb2, void *C, long ldc,
                     cudaStream_t s) {
    using CT = typename Traits<KIND>::CT;
    static const bool one_sm = getenv("X100_GEMM_1SM") != nullptr;
    static int pairs_fit[64] = {};       // co-resident CTA pairs of the 2-SM kernel
    static bool attr_set[64] = {};
    if (!attr_set[c->device]) {
        if ((KIND != 3 && cudaFuncSetAttribute(gemm_tc_kernel<(KIND == 3 ? 1 : KIND), TE>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) ||
            cudaFuncSetAttribute(gemm_tc2_kernel<KIND, TE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 P_SMEM_BYTES) != cudaSuccess)
            return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (c->sm_count / 2));
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, gemm_tc2_kernel<KIND, TE>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            nclusters = 0;
        }
        pairs_fit[c->device] = nclusters;
        attr_set[c->device] = true;
    }
    const int pair_tiles = ((M + 2 * P_ROWS - 1) / (2 * P_ROWS)) * ((N + 2 * P_COLS - 1) / (2 * P_COLS));
    if (!one_sm && pairs_fit[c->device] > 0) {
        // stream-K tail only where the partial sums are exact: int32 C updated
        // by TMA reduce-add (X100_GEMM_NO_STREAMK=1 keeps whole tiles)
        static const bool no_sk = getenv("X100_GEMM_NO_STREAMK") != nullptr;
        const int sk = (KIND == 0 && TE && !no_sk) ? 1 : 0;
        const int num_kb = (K + 127 / Traits<KIND>::ES) / (128 / Traits<KIND>::ES);
        const int fit = pairs_fit[c->device];
        int pairs = pair_tiles < fit ? pair_tiles : fit;
        if (sk && sk_pairs(pair_tiles, num_kb, fit) > 0) pairs = fit;
        // fp32 kind: K-pieces of at most X100_GEMM_F32_KPIECE k (default 1024:
        // relative error vs fp64 7.2e-6 whatever K (512: 3.7e-6; one
        // accumulator over K = 8192: 5.7e-5); at 8192^3 512-k pieces halve the
        // speed -- every piece adds its 256 x 256 accumulator into C)
        static const int kpiece = [] {
            const char *e = getenv("X100_GEMM_F32_KPIECE");
            const int v = e ? atoi(e) : 1024;
            return v >= 32 ? v : 1024;
        }();
        // fp16 -> fp32: pieces of 4096 k (relative error vs fp64 measured 4.9e-6 at
        // K = 4096 and 9.7e-6 at K = 8192 in one piece); int8 is exact and
        // fp16 C is rounded to fp16 anyway: one piece
        const int kp = KIND == 3 ? kpiece / (128 / Traits<KIND>::ES) : KIND == 1 ? 4096 / 64 : (1 << 30);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * pairs);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl_enabled() ? 1 : 0;
        return check_cuda(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<KIND, TE>, ta, tb, tc_, ta2, tb2,
                                             reinterpret_cast<CT *>(C), M, N, K, ldc, sk, kp, c->d_status),
                          X100_E_LAUNCH);
    }
    if constexpr (KIND == 3) {   // the 3-product form exists only as a 2-SM kernel
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < c->sm_count ? tiles : c->sm_count;
    constexpr int K1 = KIND == 3 ? 1 : KIND;   // not reached for kind 3
    gemm_tc_kernel<K1, TE><<<grid, THREADS, SMEM_BYTES, s>>>(ta, tb, tc_, reinterpret_cast<typename Traits<K1>::CT *>(C),
                                                            M, N, K, ldc, c->d_status);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

template <int KIND>
static int launch_kind(DevCtx *c, int M, int N, int K, const void *A, long lda, const void *B, long ldb, void *C,
                       long ldc, cudaStream_t s, const void *A2 = nullptr, const void *B2 = nullptr) {
    constexpr int ES = Traits<KIND>::ES;
    constexpr int BK = 128 / ES;
    constexpr int ATOM_N = 128 / ES;
    const CUtensorMapDataType dt = (KIND == 0)   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : (KIND == 3) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap ta, tb, tcm, ta2, tb2;
    // boxes: A BK x 128 rows, B ATOM_N columns x BK rows (the 2-SM kernel
    // loads one 128-column half of B per CTA in 128 / ATOM_N boxes); kind 3:
    // B is given transposed (N x K, row stride ldb) and boxed like A
    if (!make_tmap_2d(&ta, A, dt, (uint64_t)K, (uint64_t)M, (uint64_t)lda * ES, BK, BM) ||
        !(KIND == 3 ? make_tmap_2d(&tb, B, dt, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * ES, BK, P_COLS)
                    : make_tmap_2d(&tb, B, dt, (uint64_t)N, (uint64_t)K, (uint64_t)ldb * ES, ATOM_N, BK))) {
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    if constexpr (KIND == 3) {   // the low parts, same layouts
        if (!make_tmap_2d(&ta2, A2, dt, (uint64_t)K, (uint64_t)M, (uint64_t)lda * ES, BK, BM) ||
            !make_tmap_2d(&tb2, B2, dt, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * ES, BK, P_COLS)) {
            set_error(X100_E_UNSUPPORTED);
            return X100_E_UNSUPPORTED;
        }
    } else {
        ta2 = ta;   // unused by the kernel
        tb2 = tb;
    }
    // 32-bit C: 32 x 32 boxes added by TMA reduce-add when the layout allows
    bool te = false;
    if (KIND != 2 && reinterpret_cast<uintptr_t>(C) % 16 == 0 && (ldc * 4) % 16 == 0 && !getenv("X100_GEMM_LSU_EPI"))
        te = make_tmap_2d(&tcm, C, KIND == 0 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          (uint64_t)N, (uint64_t)M, (uint64_t)ldc * 4, 32, 32);
    if (!te) tcm = ta;   // unused by the kernel
    if constexpr (KIND != 2) {
        if (te) return launch_te<KIND, true>(c, M, N, K, ta, tb, tcm, ta2, tb2, C, ldc, s);
    }
    return launch_te<KIND, false>(c, M, N, K, ta, tb, tcm, ta2, tb2, C, ldc, s);
}

// X = X_hi + X_lo with X_hi = X rounded to tf32 (10 mantissa bits, nearest,
// ties away from zero) and X_lo = X - X_hi, exact in fp32.  X_hi is stored
// explicitly, so the products do not depend on how the tensor core reduces
// an fp32 operand to tf32 (X_hi is already a tf32 value; X_lo only loses
// bits 2^-11 below its own size).
__device__ __forceinline__ float tf32_hi(float v) {
    const uint32_t u = __float_as_uint(v);
    if ((u & 0x7F800000u) == 0x7F800000u) return v;   // inf, nan
    return __uint_as_float((u + 0x1000u) & 0xFFFFE000u);
}
__global__ void split_tf32_kernel(const float *__restrict__ x, float *__restrict__ hi, float *__restrict__ lo,
                                  long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const float v = x[i], h = tf32_hi(v);
        hi[i] = h;
        lo[i] = v - h;
    }
}
// bt[n][k] = hi(b[k][n]) and btlo[n][k] = lo(b[k][n]) for k < K, n < N
// (row strides ldb and ldt); 32 x 32 tiles through shared memory, grid
// (ceil(N/32), ceil(K/32)), block 32 x 8.
__global__ void transpose_split_kernel(const float *__restrict__ b, long ldb, int K, int N, float *__restrict__ bt,
                                       float *__restrict__ btlo, long ldt) {
    __shared__ float t[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        t[r][threadIdx.x] = (k < K && n < N) ? b[(long)k * ldb + n] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K) {
            const float v = t[threadIdx.x][r], h = tf32_hi(v);
            bt[(long)n * ldt + k] = h;
            btlo[(long)n * ldt + k] = v - h;
        }
    }
}

}  // namespace tc

bool tc_operands_ok(int kind, const void *A, long lda, const void *B, long ldb) {
    const int es = kind == 0 ? 1 : (kind == 3 ? 4 : 2);
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
    case 3: {
        // A_hi, A_lo, B^T_hi and B^T_lo in stream-ordered scratch (freed once
        // the GEMM has run): every operand of the three products is K-major
        const long na = (long)(M - 1) * lda + K, nap = (na + 3) & ~3L;
        const long ldt = (K + 3) & ~3L;   // 16-byte rows
        const long nt = (long)N * ldt;
        float *scr = nullptr;
        if (check_cuda(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&scr), (size_t)(2 * nap + 2 * nt) * 4,
                                               c->pool, s),
                       X100_E_ALLOC))
            return X100_E_ALLOC;
        float *ahi = scr, *alo = scr + nap, *bt = scr + 2 * nap, *bt2 = bt + nt;
        int st = tf32_split(c, static_cast<const float *>(A), na, ahi, alo, s);
        if (!st) st = tf32_split_transpose(c, static_cast<const float *>(B), ldb, K, N, bt, bt2, ldt, s);
        if (!st) st = launch_gemm_tf32x3(c, M, N, K, ahi, alo, lda, bt, bt2, ldt, static_cast<float *>(C), ldc, s);
        cudaFreeAsync(scr, s);
        return st;
    }
    default: set_error(X100_E_ARG); return X100_E_ARG;
    }
}

int tf32_split(DevCtx *c, const float *x, long n, float *hi, float *lo, cudaStream_t s) {
    tc::split_tf32_kernel<<<c->sm_count * 4, 256, 0, s>>>(x, hi, lo, n);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int tf32_split_transpose(DevCtx *c, const float *B, long ldb, int K, int N, float *bt, float *btlo, long ldt,
                         cudaStream_t s) {
    (void)c;
    tc::transpose_split_kernel<<<dim3((N + 31) / 32, (K + 31) / 32), dim3(32, 8), 0, s>>>(B, ldb, K, N, bt, btlo,
                                                                                       ldt);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_gemm_tf32x3(DevCtx *c, int M, int N, int K, const float *ahi, const float *alo, long lda, const float *bt,
                       const float *btlo, long ldt, float *C, long ldc, cudaStream_t s) {
    if (c->cc_major != 10) {
        set_error(X100_E_ARCH);
        return X100_E_ARCH;
    }
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    return tc::launch_kind<3>(c, M, N, K, ahi, lda, bt, ldt, C, ldc, s, alo, btlo);
}

}  // namespace x100
