// fp32-accurate GEMM on the 5th-generation tensor cores (sm_100a): 3xTF32.
//
// The tensor core reads a float32 operand as tf32 by dropping its low 13 mantissa
// bits (verified bitwise on B200: feeding x or its truncation gives identical
// products).  Each operand x is split into hi = trunc_tf32(x) and
// lo = trunc_tf32(x - hi) (x - hi is exact in fp32); C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi,
// and the dropped A_lo.B_lo term and the truncation of lo are O(2^-20) relative.
// Both halves are stored with their low 13 bits already zero although the tensor core
// would ignore them: on B200 the MMA main loop runs 6-10% faster on such operands
// than on full-mantissa fp32 (same products; less switching under the power limit).
//
// Accumulation: the tensor core's fp32 accumulation does not round to nearest (its
// error grows with the number of accumulation steps; measured ~7e-9 * K relative on
// B200), so TMEM only accumulates CHUNKS of `chunk_kb` K blocks (256 values of K by
// default).  Two TMEM accumulators (2 x 256 columns) alternate: while the MMA issuer
// fills one chunk, eight epilogue warps drain the previous one into fp32 registers
// with round-to-nearest adds.  The product then meets the 1e-5 relative-Frobenius
// contract against the reference's fp32 matmul (src/core/operators.cpp:235-319) at
// any K.
//
// Operand layout: hi and lo are written K-major (K contiguous, rows padded to 4
// floats so TMA rows are 16-B aligned) whatever the view's strides; an M- or N-major
// view is transposed through shared memory on the way.  (tcgen05 also reads
// M/N-major tf32 tiles, in the 32-B-atom 128-B swizzle, but measured ~4% slower in
// the main loop than K-major tiles, which outweighs the transposing copy.)
//
// Pipeline (one 128x256 output tile per CTA, 320 threads):
//   split pre-pass : hi/lo of both operands in scratch (vectorised rows, or 32 x 128
//                    shared-memory transposes for M/N-major views);
//   warp 0         : TMA producer, STAGES x (A_hi, A_lo, B_hi, B_lo) swizzled tiles of
//                    BK floats along K, completion on mbarriers;
//   warp 1         : allocates 512 TMEM columns; one elected thread issues
//                    tcgen05.mma.kind::tf32 (M=128, N=256, K=8; 3 products per step);
//                    tcgen05.commit frees smem stages and publishes finished chunks;
//   warps 2..9     : drain chunks (tcgen05.ld 32 lanes x 32 columns), keep the row's
//                    128 columns in registers, store to C (or to a split-K partial).
// Split-K (ksplit > 1, when the tile grid would leave the last wave of CTAs part-empty
// or the GPU under-filled; chosen by gemm_tc_plan's wave model): CTA z handles a contiguous
// range of K blocks and writes a partial tile; a reduce kernel sums the partials in
// split order (deterministic) and applies the epilogue.
// No TMA multicast: every CTA loads its own tiles (the kernel also runs inside
// multi-GPU jobs).  Every mbarrier wait is bounded by a clock budget; on expiry the
// kernel records a code in the program's status word, raises a CTA-wide abort flag
// (other CTAs see the status word and stop too), waits (bounded) for its own copies
// in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "jit.hpp"
#include "program.hpp"

namespace ttb {

namespace {

constexpr int BM = 128, BN = 256;
constexpr uint32_t TMEM_COLS = 512;                    // two 256-column accumulators
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;           // 320
constexpr long long WAIT_BUDGET = 4000000000LL;        // ~2 s of SM clock

template <int BK>
struct Cfg {
    static constexpr int STAGES = 64 / BK;                       // 2 x 96 KB or 4 x 48 KB
    static constexpr int A_TILE = BM * BK * 4;
    static constexpr int B_TILE = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 2048;
    static constexpr uint32_t KROW = BK * 4;                     // K-major row bytes: 128 or 64
    static constexpr uint32_t KLAYOUT = BK == 32 ? 2u : 4u;      // descriptor SWIZZLE_128B / SWIZZLE_64B
};

enum : int { ST_TIMEOUT_EMPTY = 0x100, ST_TIMEOUT_FULL = 0x200, ST_TIMEOUT_TFULL = 0x300, ST_TIMEOUT_TEMPTY = 0x400 };

struct TcParams {
    float* C;            // output, or the split-K partial buffer
    int64_t ldc, c_bstride;
    int M, N, K;
    int a_batched, b_batched;
    int ksplit, kb_per_split, chunk_kb;
    int tiles_m, tiles_n, n_units;  // pair kernel: 256x256 tiles and work units (tiles x batch x splits)
    int group_m;                    // pair kernel: M-tiles per group of the unit order (see pair_unit)
    // pair kernel tail split (tail_split > 0, ksplit 1): units >= n_full are pieces of the
    // last tiles, tail_kb K blocks each, written to tail_part[piece][256][256]
    int n_full, tail_split, tail_kb;
    float* tail_part;
    int epilogue;        // applied here only when ksplit == 1
    int* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false if the phase does not complete within the clock budget, if this
// CTA has aborted, or if another CTA has already reported a timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int code, long long budget = WAIT_BUDGET) {
    const long long t0 = clock64();
    uint32_t polls = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if ((++polls & 255u) == 0 && *reinterpret_cast<volatile int*>(status) != 0) {
            *abort_flag = 1;
            return false;
        }
        if (clock64() - t0 > budget) {
            *abort_flag = 1;
            atomicCAS(status, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Shared-memory matrix descriptor (sm_100 version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(layout) << 61;
    return d;
}

// Descriptor of MMA k-step `ks` (8 tf32 of K) of a K-major operand tile: rows of BK
// floats (BK*4 bytes), 8-row swizzle atoms (SBO); step = 32 B along the row.
template <int BK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, int ks) {
    return smem_desc(tile + static_cast<uint32_t>(ks) * 32u, 16u, 8u * Cfg<BK>::KROW, Cfg<BK>::KLAYOUT);
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                            (static_cast<uint32_t>(BM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BK>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                   const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo, TcParams p) {
    using C_ = Cfg<BK>;
    constexpr int STAGES = C_::STAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C_::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2] chunk accumulated  (MMA -> epilogue)
    uint64_t* tempty = tfull + 2;       // [2] chunk drained      (epilogue -> MMA)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int zb_all = blockIdx.z;
    const int batch = zb_all / p.ksplit, split = zb_all - batch * p.ksplit;
    const int za = p.a_batched ? batch : 0, zb = p.b_batched ? batch : 0;
    const int nkb_total = (p.K + BK - 1) / BK;
    const int kb0 = split * p.kb_per_split;
    const int kcount = max(0, min(nkb_total, kb0 + p.kb_per_split) - kb0);
    const int nchunks = (kcount + p.chunk_kb - 1) / p.chunk_kb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EPI_WARPS);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_ahi)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_bhi)) : "memory");
            int issued = 0;
            for (int i = 0; i < kcount; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (i / STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ST_TIMEOUT_EMPTY)) break;
                uint8_t* st = tiles + s * C_::STAGE_BYTES;
                const int kx = (kb0 + i) * BK;
                mbar_expect_tx(&full[s], C_::STAGE_BYTES);
                tma_load_3d(st, &tm_ahi, &full[s], kx, m0, za);
                tma_load_3d(st + C_::A_TILE, &tm_alo, &full[s], kx, m0, za);
                tma_load_3d(st + 2 * C_::A_TILE, &tm_bhi, &full[s], kx, n0, zb);
                tma_load_3d(st + 2 * C_::A_TILE + C_::B_TILE, &tm_blo, &full[s], kx, n0, zb);
                issued = i + 1;
            }
            if (*abort_flag) {
                // let the copies already issued land before this CTA's shared memory goes away
                for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && clock64() - t0 < WAIT_BUDGET) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int i = 0; i < kcount; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (i / STAGES) & 1;
                const int c = i / p.chunk_kb, within = i - c * p.chunk_kb;
                const int b = c & 1;
                if (within == 0) {
                    if (!mbar_wait(&tempty[b], ((c >> 1) & 1) ^ 1, abort_flag, p.status, ST_TIMEOUT_TEMPTY)) break;
                }
                if (!mbar_wait(&full[s], ph, abort_flag, p.status, ST_TIMEOUT_FULL)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t acc = tmem + static_cast<uint32_t>(b * 256);
                const uint32_t st = smem_u32(tiles + s * C_::STAGE_BYTES);
                const uint32_t ahi = st, alo = st + C_::A_TILE, bhi = st + 2 * C_::A_TILE;
                const uint32_t blo = st + 2 * C_::A_TILE + C_::B_TILE;
#pragma unroll
                for (int k = 0; k < BK / 8; ++k) {
                    const uint64_t dah = operand_desc<BK>(ahi, k), dal = operand_desc<BK>(alo, k);
                    const uint64_t dbh = operand_desc<BK>(bhi, k), dbl = operand_desc<BK>(blo, k);
                    mma_tf32(acc, dah, dbh, kIdesc, (within | k) != 0);
                    mma_tf32(acc, dah, dbl, kIdesc, 1u);
                    mma_tf32(acc, dal, dbh, kIdesc, 1u);
                }
                mma_commit(&empty[s]);
                if (within == p.chunk_kb - 1 || i == kcount - 1) mma_commit(&tfull[b]);
            }
        }
        __syncwarp();
    } else {
        // epilogue warp e (0..7): TMEM lanes 32*(warp%4).., columns 128*(e/4) .. +127
        const int e = warp - 2, q = warp & 3, h = e >> 2;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        float acc[128];
#pragma unroll
        for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int c = 0; c < nchunks; ++c) {
            const int b = c & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (c >> 1) & 1, abort_flag, p.status, ST_TIMEOUT_TFULL));
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t r[32];
                tmem_ld32(tmem + lane_base + static_cast<uint32_t>(b * 256 + h * 128 + j * 32), r);
#pragma unroll
                for (int t = 0; t < 32; ++t) acc[j * 32 + t] = __fadd_rn(acc[j * 32 + t], __uint_as_float(r[t]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
        }
        if (ok) {
            const int row = m0 + q * 32 + lane;
            float* crow = p.C + static_cast<int64_t>(zb_all) * p.c_bstride + static_cast<int64_t>(row) * p.ldc;
            const bool vec_ok = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                                (p.c_bstride % 4 == 0);
            if (row < p.M) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col0 = n0 + h * 128 + j * 32;
                    if (col0 < p.N) {
                        float v[32];
#pragma unroll
                        for (int t = 0; t < 32; ++t) {
                            v[t] = gemm_epilogue(acc[j * 32 + t], p.epilogue);
                        }
                        if (vec_ok && col0 + 32 <= p.N) {
#pragma unroll
                            for (int t = 0; t < 32; t += 4)
                                *reinterpret_cast<float4*>(crow + col0 + t) =
                                    make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
                        } else {
#pragma unroll
                            for (int t = 0; t < 32; ++t)
                                if (col0 + t < p.N) crow[col0 + t] = v[t];
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// ---- CTA-pair variant (tcgen05 cta_group::2): 256 x 256 output tile per 2-CTA cluster ----
// CTA rank r of the pair holds rows [128r, 128r+128) of the A tile and rows [128r, 128r+128)
// of the 256-row B tile in its own shared memory, at the same offsets in both CTAs.  The
// even CTA (the leader) issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 8): the
// tensor cores of both SMs read A and B from both CTAs' shared memory and CTA r's TMEM
// receives output rows [128r, 128r+128) x 256 columns.  Compared with one CTA per
// 128x256 tile, each SM stores and reads half as many B bytes per K block, which is what
// bounds the single-CTA main loop (shared-memory bandwidth).
// Barriers: both CTAs' TMA loads complete on the LEADER's full[s] (the leader expects the
// pair's bytes); the leader's commits arrive on empty[s] / tfull[b] in both CTAs (one
// commit per CTA, the peer's barrier addressed through mapa); the epilogue warps of both
// CTAs arrive on the leader's tempty[b] (16 arrivals).  Every wait is bounded as in the
// single-CTA kernel, and both CTAs meet at a cluster barrier before TMEM is freed and
// before either exits, so no arrival targets a CTA that has left.
constexpr int PAIR_STAGES = 3;

template <int BK>
struct PairCfg {
    static constexpr int TILE = 128 * BK * 4;               // 128 rows x BK floats (A or B half)
    static constexpr int STAGE_BYTES = 4 * TILE;            // A_hi, A_lo, B_hi, B_lo of this CTA
    static constexpr int SMEM_BYTES = PAIR_STAGES * STAGE_BYTES + 2048;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of this CTA's shared variable `p` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on a barrier that receives arrivals from the peer CTA (cluster acquire).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* status, int code) {
    const long long t0 = clock64();
    uint32_t polls = 0;
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (*abort_flag) return false;
        if ((++polls & 255u) == 0 && *reinterpret_cast<volatile int*>(status) != 0) {
            *abort_flag = 1;
            return false;
        }
        if (clock64() - t0 > WAIT_BUDGET) {
            *abort_flag = 1;
            atomicCAS(status, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrives on the barrier at cluster address `bar` when this thread's MMAs complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 256 (the pair), N = 256.
constexpr uint32_t kIdescPair = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(256 >> 3) << 17) |
                                (static_cast<uint32_t>(256 >> 4) << 24);

// Work unit u of the persistent pair kernel: output pair-tile (tm, tn) of batch/split zz.
// Within a batch/split the tiles are taken in groups of group_m M-tiles: inside a group
// M-tiles vary fastest, then N-tiles, and every other group walks its N-tiles backwards.
// The clusters running at one time hold consecutive units, so they cover a block of
// about group_m x (clusters / group_m) tiles instead of a few whole rows of tiles: fewer
// A and B panels are streamed at once (each read from DRAM once and shared through L2
// by the tiles of its row or column), and the B panels at the turn between two groups
// are still in L2.  group_m = 1 walks rows of tiles (N-tiles fastest), alternating
// direction.
// Tail split (tail_split = S > 0): when the tiles leave the last round of clusters part
// full (r = T mod clusters tiles), units [0, n_full) are whole tiles as above and units
// n_full + v (v < r * S) are piece v % S of tile n_full + v / S: K blocks
// [piece * tail_kb, +tail_kb), stored without activation as a partial tile
// tail_part[v][256][256].  Each cluster of the last round then takes one piece, so that
// round lasts about 1/S of a tile instead of a whole one; tail_reduce_kernel adds the S
// partials of each tile in piece order and applies the activation.
struct PairUnit {
    int n0, m0, nb0, zb_all, za, zb, kb0, kcount, piece;
};

struct PairTile {
    int tm, tn, zz;
};

// Tile t of the raster order described above (zz = batch, or batch * ksplit + split).
__device__ __forceinline__ PairTile pair_tile(int tiles_m, int tiles_n, int group_m, int t) {
    PairTile r;
    const int per_z = tiles_m * tiles_n;
    r.zz = t / per_z;
    const int rem = t - r.zz * per_z;
    const int span = group_m * tiles_n;  // units of a full group
    const int g = rem / span, first = g * group_m;
    const int gsz = min(group_m, tiles_m - first);
    const int i = rem - g * span;
    r.tm = first + i % gsz;
    r.tn = (g & 1) ? tiles_n - 1 - i / gsz : i / gsz;
    return r;
}

__device__ __forceinline__ PairUnit pair_unit(const TcParams& p, int u, uint32_t rank, int nkb_total) {
    PairUnit w;
    int t = u;
    w.piece = -1;
    if (p.tail_split > 0 && u >= p.n_full) {
        const int v = u - p.n_full, tile = v / p.tail_split;
        t = p.n_full + tile;
        w.piece = v;
        w.kb0 = (v - tile * p.tail_split) * p.tail_kb;
        w.kcount = max(0, min(nkb_total, w.kb0 + p.tail_kb) - w.kb0);
    }
    const PairTile pt = pair_tile(p.tiles_m, p.tiles_n, p.group_m, t);
    w.n0 = pt.tn * 256;
    w.m0 = pt.tm * 256 + static_cast<int>(rank) * 128;
    w.nb0 = w.n0 + static_cast<int>(rank) * 128;
    w.zb_all = pt.zz;
    const int batch = pt.zz / p.ksplit, split = pt.zz - batch * p.ksplit;
    w.za = p.a_batched ? batch : 0;
    w.zb = p.b_batched ? batch : 0;
    if (w.piece < 0) {
        w.kb0 = split * p.kb_per_split;
        w.kcount = max(0, min(nkb_total, w.kb0 + p.kb_per_split) - w.kb0);
    }
    return w;
}

// Persistent: each cluster walks the units u = cluster, cluster + clusters, ...  The
// stage ring, the TMEM chunk double buffer and every barrier phase run on counters
// that continue across units, so the epilogue of one tile (its last drain and its
// stores) overlaps the TMA loads and MMAs of the next.
template <int BK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                        const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                        TcParams p) {
    using C_ = PairCfg<BK>;
    constexpr int STAGES = PAIR_STAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C_::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2] chunk accumulated  (leader's MMA -> both epilogues)
    uint64_t* tempty = tfull + 2;       // [2] chunk drained      (both epilogues -> leader's MMA)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
    const int nkb_total = (p.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI_WARPS);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_ahi)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_bhi)) : "memory");
            uint32_t gs = 0;  // stages issued so far (all units)
            bool stop = false;
            for (int u = cluster; u < p.n_units && !stop; u += clusters) {
                const PairUnit w = pair_unit(p, u, rank, nkb_total);
                for (int i = 0; i < w.kcount; ++i, ++gs) {
                    const int s = static_cast<int>(gs % STAGES);
                    const uint32_t ph = (gs / STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ST_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
                    uint8_t* st = tiles + s * C_::STAGE_BYTES;
                    const int kx = (w.kb0 + i) * BK;
                    if (leader) mbar_expect_tx(&full[s], 2 * C_::STAGE_BYTES);
                    const uint32_t fb = mapa_shared(&full[s], 0);
                    tma_load_3d_pair(st, &tm_ahi, fb, kx, w.m0, w.za);
                    tma_load_3d_pair(st + C_::TILE, &tm_alo, fb, kx, w.m0, w.za);
                    tma_load_3d_pair(st + 2 * C_::TILE, &tm_bhi, fb, kx, w.nb0, w.zb);
                    tma_load_3d_pair(st + 3 * C_::TILE, &tm_blo, fb, kx, w.nb0, w.zb);
                }
            }
            if (*abort_flag && gs > 0) {
                if (leader) {
                    // let the copies already issued land before shared memory goes away
                    for (uint32_t i = (gs > STAGES ? gs - STAGES : 0); i < gs; ++i) {
                        const long long t0 = clock64();
                        while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && clock64() - t0 < WAIT_BUDGET) {
                        }
                    }
                } else {
                    // the follower's copies complete on the leader's barrier: give them time
                    const long long t0 = clock64();
                    while (clock64() - t0 < WAIT_BUDGET / 4) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            uint32_t gs = 0, gc = 0;  // stages consumed, chunks accumulated (all units)
            bool stop = false;
            for (int u = cluster; u < p.n_units && !stop; u += clusters) {
                const PairUnit w = pair_unit(p, u, rank, nkb_total);
                for (int i = 0; i < w.kcount; ++i, ++gs) {
                    const int s = static_cast<int>(gs % STAGES);
                    const uint32_t ph = (gs / STAGES) & 1;
                    const int within = i % p.chunk_kb;
                    const int b = static_cast<int>(gc & 1);
                    if (within == 0 &&
                        !mbar_wait_cluster(&tempty[b], ((gc >> 1) & 1) ^ 1, abort_flag, p.status, ST_TIMEOUT_TEMPTY)) {
                        stop = true;
                        break;
                    }
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ST_TIMEOUT_FULL)) {
                        stop = true;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t acc = tmem + static_cast<uint32_t>(b * 256);
                    const uint32_t st = smem_u32(tiles + s * C_::STAGE_BYTES);
                    const uint32_t ahi = st, alo = st + C_::TILE, bhi = st + 2 * C_::TILE, blo = st + 3 * C_::TILE;
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {
                        const uint64_t dah = operand_desc<BK>(ahi, k), dal = operand_desc<BK>(alo, k);
                        const uint64_t dbh = operand_desc<BK>(bhi, k), dbl = operand_desc<BK>(blo, k);
                        mma_tf32_pair(acc, dah, dbh, kIdescPair, (within | k) != 0);
                        mma_tf32_pair(acc, dah, dbl, kIdescPair, 1u);
                        mma_tf32_pair(acc, dal, dbh, kIdescPair, 1u);
                    }
                    mma_commit_pair(mapa_shared(&empty[s], 0));
                    mma_commit_pair(mapa_shared(&empty[s], 1));
                    if (within == p.chunk_kb - 1 || i == w.kcount - 1) {
                        mma_commit_pair(mapa_shared(&tfull[b], 0));
                        mma_commit_pair(mapa_shared(&tfull[b], 1));
                        ++gc;
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // epilogue warp e (0..7): TMEM lanes 32*(warp%4).., columns 128*(e/4) .. +127
        const int e = warp - 2, q = warp & 3, h = e >> 2;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const bool vec_ok = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                            (p.c_bstride % 4 == 0);
        uint32_t ec = 0;  // chunks drained (all units)
        bool ok = true;
        for (int u = cluster; u < p.n_units && ok; u += clusters) {
            const PairUnit w = pair_unit(p, u, rank, nkb_total);
            const int nchunks = (w.kcount + p.chunk_kb - 1) / p.chunk_kb;
            float acc[128];
#pragma unroll
            for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
            for (int c = 0; c < nchunks; ++c, ++ec) {
                const int b = static_cast<int>(ec & 1);
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&tfull[b], (ec >> 1) & 1, abort_flag, p.status, ST_TIMEOUT_TFULL));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t r[32];
                    tmem_ld32(tmem + lane_base + static_cast<uint32_t>(b * 256 + h * 128 + j * 32), r);
#pragma unroll
                    for (int t = 0; t < 32; ++t) acc[j * 32 + t] = __fadd_rn(acc[j * 32 + t], __uint_as_float(r[t]));
                }
                asm volatile("tcgen05.fence::before_thread_sync;");
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(&tempty[b], 0));
            }
            if (!ok) break;
            const int row = w.m0 + q * 32 + lane;
            // row `row` from column w.n0 on: in C, or in this piece's partial tile
            const bool part = w.piece >= 0;
            float* crow = part ? p.tail_part + (static_cast<int64_t>(w.piece) * 256 + (w.m0 & 255) + q * 32 + lane) * 256
                               : p.C + static_cast<int64_t>(w.zb_all) * p.c_bstride + static_cast<int64_t>(row) * p.ldc +
                                     w.n0;
            const int ep = part ? EP_NONE : p.epilogue;
            if (row < p.M) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col0 = w.n0 + h * 128 + j * 32;
                    if (col0 < p.N) {
                        float v[32];
#pragma unroll
                        for (int t = 0; t < 32; ++t) {
                            v[t] = gemm_epilogue(acc[j * 32 + t], ep);
                        }
                        float* dst = crow + (col0 - w.n0);
                        if ((vec_ok || part) && col0 + 32 <= p.N) {
#pragma unroll
                            for (int t = 0; t < 32; t += 4)
                                *reinterpret_cast<float4*>(dst + t) = make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
                        } else {
#pragma unroll
                            for (int t = 0; t < 32; ++t)
                                if (col0 + t < p.N) dst[t] = v[t];
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    cluster_sync_all();  // all MMAs done, all remote arrivals delivered, in both CTAs
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// Sums split-K partials P[b][s][i] in split order and applies the epilogue.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ P, float* __restrict__ C,
                                                            int64_t per, int ksplit, int64_t c_bstride, int epilogue) {
    const int64_t b = blockIdx.y;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * 256;
    const bool vec = (per % 4 == 0) && (c_bstride % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    if (vec) {
        // float4 per thread; the ksplit loads of one float4 are independent (in flight together)
        for (int64_t i = (static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x) * 4; i < per; i += stride * 4) {
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int s = 0; s < ksplit; ++s) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(P + (b * ksplit + s) * per + i));
                v.x = __fadd_rn(v.x, x.x);
                v.y = __fadd_rn(v.y, x.y);
                v.z = __fadd_rn(v.z, x.z);
                v.w = __fadd_rn(v.w, x.w);
            }
            v.x = gemm_epilogue(v.x, epilogue);
            v.y = gemm_epilogue(v.y, epilogue);
            v.z = gemm_epilogue(v.z, epilogue);
            v.w = gemm_epilogue(v.w, epilogue);
            *reinterpret_cast<float4*>(C + b * c_bstride + i) = v;
        }
        return;
    }
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < per; i += stride) {
        float v = 0.0f;
        for (int s = 0; s < ksplit; ++s) v = __fadd_rn(v, __ldg(P + (b * ksplit + s) * per + i));
        C[b * c_bstride + i] = gemm_epilogue(v, epilogue);
    }
}

// Adds the S partial tiles of each tail tile of the pair kernel (its tail split) in piece
// order, applies the epilogue and stores the tile's in-range part of C.  Grid:
// (16, tail tiles); a thread handles 4 consecutive columns of a row per step.
__global__ void __launch_bounds__(256) tail_reduce_kernel(const float* __restrict__ P, float* __restrict__ C, int M,
                                                          int N, int64_t ldc, int64_t c_bstride, int tiles_m,
                                                          int tiles_n, int group_m, int n_full, int S, int epilogue) {
    const int i = blockIdx.y;
    const PairTile pt = pair_tile(tiles_m, tiles_n, group_m, n_full + i);
    const bool vec = (ldc % 4 == 0) && (c_bstride % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    for (int e = blockIdx.x * 256 + threadIdx.x; e < 256 * 64; e += gridDim.x * 256) {
        const int lr = e >> 6, lc = (e & 63) * 4;
        const int row = pt.tm * 256 + lr, col = pt.tn * 256 + lc;
        if (row >= M || col >= N) continue;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int s = 0; s < S; ++s) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(P + ((static_cast<int64_t>(i) * S + s) * 256 + lr) * 256 + lc));
            v.x = __fadd_rn(v.x, x.x);
            v.y = __fadd_rn(v.y, x.y);
            v.z = __fadd_rn(v.z, x.z);
            v.w = __fadd_rn(v.w, x.w);
        }
        v.x = gemm_epilogue(v.x, epilogue);
        v.y = gemm_epilogue(v.y, epilogue);
        v.z = gemm_epilogue(v.z, epilogue);
        v.w = gemm_epilogue(v.w, epilogue);
        float* out = C + static_cast<int64_t>(pt.zz) * c_bstride + static_cast<int64_t>(row) * ldc + col;
        if (vec && col + 4 <= N) {
            *reinterpret_cast<float4*>(out) = v;
        } else {
            const float q[4] = {v.x, v.y, v.z, v.w};
            for (int t = 0; t < 4 && col + t < N; ++t) out[t] = q[t];
        }
    }
}

// ---- split pre-pass ----
// hi = trunc_tf32(x), lo = trunc_tf32(x - hi) (x - hi is exact in fp32).
// Non-finite products follow the reference's fp32 loop (src/core/operators.cpp:235-319),
// where a.b is +-inf for a = +-inf and any finite nonzero b, and NaN for inf * 0.  In
// C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi a zero lo part next to an infinite partner
// would add an inf * 0 = NaN term, so lo is never zero for a nonzero x:
//   - x nonzero and tf32-exact (x - hi == 0): lo = hi * 2^-24, a marker of x's sign
//     (it moves the represented value by 2^-24 relative, below the scheme's 2^-21);
//   - x = +-inf: hi = lo = x;  NaN: hi = lo = the canonical quiet NaN (its payload
//     survives the truncation);  x = +-0: hi = x, lo = +0.
// Then every product term with an infinite factor is inf of the right sign (or NaN
// for inf * 0, as in the reference), and sums of them behave as the reference's.  The
// marker underflows only for |x| < 2^-102 (then an inf partner gives NaN, not inf).
__device__ __forceinline__ float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    if (isfinite(x)) {
        hi = trunc_tf32(x);
        const float r = trunc_tf32(__fsub_rn(x, hi));
        lo = (r == 0.0f && x != 0.0f) ? trunc_tf32(__fmul_rn(hi, 0x1p-24f)) : r;
    } else {
        hi = isnan(x) ? __uint_as_float(0x7FC00000u) : x;
        lo = hi;
    }
}

// View X[b][r][k] = X[b*s_b + r*s_r + k*s_k] -> hi/lo[b*l_b + r*l_r + k].  Work units
// are 1024-float segments of a row, one warp per unit (so a few long rows still spread
// over the whole GPU); the vec4 path (s_k == 1, K % 4 == 0, X, s_r and s_b 16-B
// aligned) issues a lane's eight float4 loads before its stores, 4 KB in flight per warp.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ X, float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t R, int64_t K, int64_t s_r,
                                                         int64_t s_k, int64_t s_b, int64_t l_r, int64_t l_b,
                                                         int vec4) {
    constexpr int SEG = 1024;
    const int64_t b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* xb = X + b * s_b;
    const int64_t segs = (K + SEG - 1) / SEG;
    for (int64_t u = static_cast<int64_t>(blockIdx.x) * 8 + warp; u < R * segs; u += static_cast<int64_t>(gridDim.x) * 8) {
        const int64_t r = u / segs, k0 = (u - r * segs) * SEG;
        const int64_t k1 = k0 + SEG < K ? k0 + SEG : K;
        const float* xr = xb + r * s_r;
        float* hr = hi + b * l_b + r * l_r;
        float* lr = lo + b * l_b + r * l_r;
        if (vec4) {
            float4 x[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int64_t i = k0 + lane * 4 + 128 * j;
                x[j] = i < k1 ? __ldg(reinterpret_cast<const float4*>(xr + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int64_t i = k0 + lane * 4 + 128 * j;
                if (i >= k1) break;
                float4 h, l;
                split_tf32(x[j].x, h.x, l.x);
                split_tf32(x[j].y, h.y, l.y);
                split_tf32(x[j].z, h.z, l.z);
                split_tf32(x[j].w, h.w, l.w);
                *reinterpret_cast<float4*>(hr + i) = h;
                *reinterpret_cast<float4*>(lr + i) = l;
            }
        } else {
            for (int64_t i = k0 + lane; i < k1; i += 32) split_tf32(__ldg(xr + i * s_k), hr[i], lr[i]);
        }
    }
}

// M/N-contiguous view (s_r == 1) -> K-major hi/lo[b*l_b + r*l_r + k]: the source is
// read as a row-major [K][R] matrix (row stride s_k) in tiles of 32 K-rows x 128 R-columns,
// one CTA per tile.  Each warp loads rows w, w+8, w+16, w+24 of the tile with a float4 of
// columns per lane (all four loads issued before any store) and parks them TRANSPOSED in
// shared memory, tile[r][k] with a pitch of 33 floats: lane l's four values go to rows
// 4l..4l+3, and the lanes of octet j store their value j first, so one store instruction
// hits 32 distinct banks.  Then lane (rs = l / 8, k4 = l % 8) of warp w takes rows
// r = 16w + 4i + rs (i < 4) and reads k = 4k4..4k4+3 of each (banks rs + 4k4 + k - 4k4:
// distinct), splits the four values and writes hi and lo as one float4 each: a warp's
// store covers 4 rows x 128 B.  Tiles are numbered K first, so the CTAs resident together
// extend the same hi/lo rows.  vec4 (R % 4 == 0, X, s_k and s_b 16-B aligned) allows the
// float4 loads; the float4 stores need l_r % 4 == 0 (always: rows are padded to 4) and a
// tile whose four k's are all inside K, else scalar stores.  Only k < K is written (the
// rows' padding up to l_r is never read).
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ X, float* __restrict__ hi,
                                                              float* __restrict__ lo, int64_t R, int64_t K,
                                                              int64_t s_k, int64_t s_b, int64_t l_r, int64_t l_b,
                                                              int vec4) {
    __shared__ float tile[128][33];
    const int64_t b = blockIdx.y;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t tiles_k = (K + 31) / 32;
    const int64_t k0 = (static_cast<int64_t>(blockIdx.x) % tiles_k) * 32;
    const int64_t r0 = (static_cast<int64_t>(blockIdx.x) / tiles_k) * 128;
    const float* xb = X + b * s_b;
    const int64_t r = r0 + 4 * lane;
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t k = k0 + w + 8 * i;
        const float* src = xb + k * s_k + r;
        if (vec4 && k < K && r < R) {
            v[i] = __ldg(reinterpret_cast<const float4*>(src));
        } else {
            v[i].x = (k < K && r < R) ? __ldg(src) : 0.0f;
            v[i].y = (k < K && r + 1 < R) ? __ldg(src + 1) : 0.0f;
            v[i].z = (k < K && r + 2 < R) ? __ldg(src + 2) : 0.0f;
            v[i].w = (k < K && r + 3 < R) ? __ldg(src + 3) : 0.0f;
        }
    }
    const int rot = lane >> 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int cc = (c + rot) & 3;  // selects, not an indexed array (which would live in local memory)
            const float e = cc == 0 ? v[i].x : cc == 1 ? v[i].y : cc == 2 ? v[i].z : v[i].w;
            tile[4 * lane + cc][w + 8 * i] = e;
        }
    }
    __syncthreads();
    const int rs = lane >> 3, k4 = lane & 7;
    const int64_t k = k0 + 4 * k4;
    const bool kfull = k + 3 < K;
    float* hb = hi + b * l_b;
    float* lb = lo + b * l_b;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rl = 16 * w + 4 * i + rs;
        const int64_t rr = r0 + rl;
        if (rr >= R) continue;
        float4 h, l;
        split_tf32(tile[rl][4 * k4], h.x, l.x);
        split_tf32(tile[rl][4 * k4 + 1], h.y, l.y);
        split_tf32(tile[rl][4 * k4 + 2], h.z, l.z);
        split_tf32(tile[rl][4 * k4 + 3], h.w, l.w);
        float* hd = hb + rr * l_r + k;
        float* ld = lb + rr * l_r + k;
        if (kfull) {
            *reinterpret_cast<float4*>(hd) = h;
            *reinterpret_cast<float4*>(ld) = l;
        } else {
            const float hv[4] = {h.x, h.y, h.z, h.w}, lv[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (k + u < K) {
                    hd[u] = hv[u];
                    ld[u] = lv[u];
                }
            }
        }
    }
}

int64_t round4(int64_t x) { return (x + 3) / 4 * 4; }
int64_t align256b(int64_t bytes) { return (bytes + 255) / 256 * 256; }

// Compact K-major hi/lo arrays of one operand (rows R along M or N, K columns):
// [nb][R][Kp], Kp = K rounded up to 4 floats so that every TMA row is 16-B aligned.
struct OperandPlan {
    int64_t nb = 1;          // batches stored (1 when broadcast over the batch)
    int64_t lr = 0, lb = 0;  // row and batch strides (elements)
};

OperandPlan plan_operand(int64_t R, int64_t K, int64_t s_b, int64_t batch) {
    OperandPlan o;
    o.nb = s_b ? batch : 1;
    o.lr = round4(K);
    o.lb = R * o.lr;
    return o;
}

int launch_split(const float* X, float* hi, float* lo, int64_t R, int64_t K, int64_t s_r, int64_t s_k, int64_t s_b,
                 const OperandPlan& o, cudaStream_t st) {
    if (R == 0 || K == 0) return 0;
    const bool x16 = (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (o.nb == 1 || s_b % 4 == 0);
    if (s_r == 1 && s_k != 1 && R > 1 && K > 1) {
        const bool vec4 = x16 && R % 4 == 0 && s_k % 4 == 0;
        const int64_t tiles = ((K + 31) / 32) * ((R + 127) / 128);  // one CTA per 32 (K) x 128 (R) tile
        if (tiles > 0x7FFFFFFFLL) return static_cast<int>(cudaErrorInvalidValue);
        split_transpose_kernel<<<dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(o.nb)), 256, 0, st>>>(
            X, hi, lo, R, K, s_k, s_b, o.lr, o.lb, vec4 ? 1 : 0);
        return static_cast<int>(cudaGetLastError());
    }
    const bool vec4 = x16 && (s_k == 1 || K == 1) && K % 4 == 0 && s_r % 4 == 0;
    static const int rows_per_sm = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, split_rows_kernel, 256, 0) != cudaSuccess) n = 4;
        return n > 0 ? n : 1;
    }();
    int64_t blocks = (R * ((K + 1023) / 1024) + 7) / 8;
    if (blocks > 148 * rows_per_sm) blocks = 148 * rows_per_sm;
    split_rows_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(o.nb)), 256, 0, st>>>(
        X, hi, lo, R, K, s_r, s_k, s_b, o.lr, o.lb, vec4 ? 1 : 0);
    return static_cast<int>(cudaGetLastError());
}

// Tensor map of one compact operand array: dims {K, R, nb}, box {bk, box_rows, 1}.
void encode_operand(CUtensorMap* map, const float* base, int64_t R, int64_t K, const OperandPlan& o, int bk,
                    int box_rows) {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(R), static_cast<cuuint64_t>(o.nb)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(o.lr * 4), static_cast<cuuint64_t>(o.lb * 4)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(bk), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUresult r = driver().tensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                                               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(TT_ERR_RUNTIME, "cuTensorMapEncodeTiled: " + cu_error(r));
}

// CTAs of one launch without split-K: one per 128x256 tile, or two per 256x256 pair tile.
int64_t ctas_of(const GemmDesc& d) {
    if (d.pair) return 2 * ((d.M + 255) / 256) * ((d.N + 255) / 256) * d.batch;
    return ((d.M + BM - 1) / BM) * ((d.N + BN - 1) / BN) * d.batch;
}

template <int BK>
int launch_main(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
                const TcParams& p, dim3 grid, cudaStream_t st) {
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        err = cudaFuncSetAttribute(gemm_tc_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg<BK>::SMEM_BYTES);
    });
    if (err != cudaSuccess) return static_cast<int>(err);
    gemm_tc_kernel<BK><<<grid, THREADS, Cfg<BK>::SMEM_BYTES, st>>>(ahi, alo, bhi, blo, p);
    return static_cast<int>(cudaGetLastError());
}

// Co-resident 2-CTA clusters of the pair kernel on the current device (the occupancy
// API; half the SM count, or 74, where it cannot be asked), with the attribute error.
template <int BK>
int pair_max_clusters(cudaError_t* attr_err) {
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    static int max_clusters = 74;
    std::call_once(once, [] {
        err = cudaFuncSetAttribute(gemm_tc_pair_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   PairCfg<BK>::SMEM_BYTES);
        if (err != cudaSuccess) return;
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(sms > 1 ? sms : 2), 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = PairCfg<BK>::SMEM_BYTES;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_pair_kernel<BK>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sms / 2 > 0 ? sms / 2 : 74;
        }
        max_clusters = n;
    });
    if (attr_err) *attr_err = err;
    return max_clusters;
}

// Persistent launch: one cluster per co-resident SM pair (at most one per work unit).
template <int BK>
int launch_pair(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
                const TcParams& p, cudaStream_t st) {
    cudaError_t err = cudaSuccess;
    const int max_clusters = pair_max_clusters<BK>(&err);
    if (err != cudaSuccess) return static_cast<int>(err);
    const int clusters = p.n_units < max_clusters ? p.n_units : max_clusters;
    if (clusters <= 0) return 0;
    gemm_tc_pair_kernel<BK><<<dim3(static_cast<unsigned>(2 * clusters)), THREADS, PairCfg<BK>::SMEM_BYTES, st>>>(
        ahi, alo, bhi, blo, p);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

bool gemm_tc_supported(const GemmDesc& d) {
    const bool big = d.M >= 64 && (d.N >= 64 || d.K >= 512);
    return big && d.K >= 1 && d.batch <= 65535 && d.M < (1LL << 31) && d.N < (1LL << 31) && d.K < (1LL << 31);
}

// Split-K choice by a wave model.  One 128x256 tile per CTA and one CTA per SM, so a
// grid of n CTAs runs in ceil(n / 148) waves; a launch whose tile count leaves the
// last wave part-empty (512 tiles = 3.46 waves) idles up to a quarter of the GPU.
// For each candidate split count ks (splits of >= one 256-K TMEM chunk) the model
// costs  waves(tiles * ks) * (K blocks per split + per-tile overhead)  plus the extra
// HBM traffic of the partials (written, then read back by the reduce), converted to
// K-block times, and keeps the cheapest.  Constants are B200 measurements: one
// 32-wide K block of a tile takes ~1.27 us (3xTF32 at ~245 TFLOP/s over 148 SMs),
// during which HBM moves ~8.3 MB.
#ifndef TT_GEMM_BK
#define TT_GEMM_BK 32
#endif
#ifndef TT_GEMM_PAIR
#define TT_GEMM_PAIR 1
#endif
#ifndef TT_GEMM_GROUP_M
#define TT_GEMM_GROUP_M 8
#endif
void gemm_tc_plan(GemmDesc& d) {
    d.bk = TT_GEMM_BK;
    d.chunk_kb = 256 / d.bk;  // 256 values of K per TMEM chunk
    d.pair = (TT_GEMM_PAIR && d.bk == 32 && d.M > 128) ? 1 : 0;
    const int64_t nkb = (d.K + d.bk - 1) / d.bk;
    const int64_t tiles = ctas_of(d);
    const double kb_us = 1.27 * d.bk / 32.0;
    const double bytes_per_kb = 6.5e12 * kb_us * 1e-6;
    const double tile_overhead_kb = 10.0;  // prologue, TMEM setup, epilogue drain and store (fitted)
    const double out_bytes = static_cast<double>(d.M) * static_cast<double>(d.N) * 4.0 * static_cast<double>(d.batch);
    int64_t best_ks = 1;
    double best_cost = 0.0;
    for (int64_t ks = 1; ks <= 16; ++ks) {
        const int64_t per = (nkb + ks - 1) / ks;
        const int64_t ks_eff = (nkb + per - 1) / per;
        if (ks_eff != ks) continue;                        // same split as a smaller ks
        if (ks > 1 && per < d.chunk_kb) break;             // splits shorter than a chunk
        if (ks * d.batch > 65535) break;
        if (ks > 1 && out_bytes * static_cast<double>(ks) > 2e9) break;  // partials' scratch
        const int64_t waves = (tiles * ks + 147) / 148;
        double cost = static_cast<double>(waves) * (static_cast<double>(per) + tile_overhead_kb);
        if (ks > 1) cost += 2.0 * static_cast<double>(ks) * out_bytes / bytes_per_kb;
        if (ks == 1 || cost < best_cost * 0.95) {         // a split must clearly pay for itself
            best_cost = cost;
            best_ks = ks;
        }
    }
    d.ksplit = static_cast<int>(best_ks);
    d.tail_tiles = d.tail_split = 0;
    // Tail split of the persistent pair kernel: with T tiles on C clusters the last round
    // holds r = T mod C tiles; splitting each of them in S = min(C / r, chunks) K pieces
    // gives every cluster of that round one piece, so it lasts ~1/S of a tile (plus the
    // pieces' partial tiles, written and read back once by the reduce).  Whole tiles keep
    // the plain epilogue.  4096^3 and 16384x1024x4096 (256 tiles on 74 clusters: 3.46
    // rounds) drop from 4 rounds to 3.5.
    if (d.pair) {
        const int64_t T = ((d.M + 255) / 256) * ((d.N + 255) / 256) * d.batch;
        const int64_t C = pair_max_clusters<32>(nullptr);
        const int64_t k = T / C, r = T - k * C;
        const int64_t nch = (nkb + d.chunk_kb - 1) / d.chunk_kb;
        int64_t S = r > 0 ? std::min<int64_t>(C / r, nch) : 0;
        if (S >= 2) {
            const int64_t per = (nkb + S - 1) / S;
            const int64_t tail_kb = (per + d.chunk_kb - 1) / d.chunk_kb * d.chunk_kb;
            S = (nkb + tail_kb - 1) / tail_kb;
            double cost = static_cast<double>(k) * (static_cast<double>(nkb) + tile_overhead_kb) +
                          static_cast<double>(tail_kb) + tile_overhead_kb;
            cost += 2.0 * static_cast<double>(r * S) * 65536.0 * 4.0 / bytes_per_kb;  // partial tiles
            if (S >= 2 && cost < best_cost * 0.95) {
                d.ksplit = 1;
                d.tail_tiles = static_cast<int>(r);
                d.tail_split = static_cast<int>(S);
            }
        }
    }
}

// Compact hi (or lo) array size of one operand, elements.
static int64_t operand_elems(int64_t R, int64_t K, int64_t s_b, int64_t batch) {
    return (s_b ? batch : 1) * R * round4(K);
}

int64_t gemm_tc_scratch_bytes(const GemmDesc& d) {
    const int64_t a = d.a_presplit ? 0 : operand_elems(d.M, d.K, d.a_sb, d.batch);
    const int64_t b = d.b_presplit ? 0 : operand_elems(d.N, d.K, d.b_sb, d.batch);
    int64_t bytes = 2 * align256b(a * 4) + 2 * align256b(b * 4);
    if (d.ksplit > 1) bytes += align256b(d.batch * d.ksplit * d.M * d.N * 4);
    if (d.tail_split > 0) bytes += align256b(static_cast<int64_t>(d.tail_tiles) * d.tail_split * 65536 * 4);
    return bytes;
}

int launch_gemm_tc(const GemmDesc& d, const float* A, const float* B, float* C, void* scratch, int* status,
                   void* stream, const GemmSplitIO* io) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const OperandPlan ap = plan_operand(d.M, d.K, d.a_sb, d.batch);
    const OperandPlan bp = plan_operand(d.N, d.K, d.b_sb, d.batch);
    if ((d.a_presplit || d.b_presplit) && (io == nullptr || d.batch != 1))
        return static_cast<int>(cudaErrorInvalidValue);  // the scheduler never plans this
    const int64_t a_cap = d.a_presplit ? 0 : align256b(operand_elems(d.M, d.K, d.a_sb, d.batch) * 4);
    const int64_t b_cap = d.b_presplit ? 0 : align256b(operand_elems(d.N, d.K, d.b_sb, d.batch) * 4);
    char* s = static_cast<char*>(scratch);
    // operand hi/lo: written into scratch by the pre-pass, or the producing region's copies
    float* ahi = d.a_presplit ? const_cast<float*>(io->a_hi) : reinterpret_cast<float*>(s);
    float* alo = d.a_presplit ? const_cast<float*>(io->a_lo) : reinterpret_cast<float*>(s + a_cap);
    float* bhi = d.b_presplit ? const_cast<float*>(io->b_hi) : reinterpret_cast<float*>(s + 2 * a_cap);
    float* blo = d.b_presplit ? const_cast<float*>(io->b_lo) : reinterpret_cast<float*>(s + 2 * a_cap + b_cap);
    float* partial = reinterpret_cast<float*>(s + 2 * a_cap + 2 * b_cap);  // split-K partials, or tail pieces
    int rc = 0;
    if (!d.a_presplit) {
        rc = launch_split(A, ahi, alo, d.M, d.K, d.a_sm, d.a_sk, d.a_sb, ap, st);
        if (rc) return rc;
    }
    if (!d.b_presplit) {
        rc = launch_split(B, bhi, blo, d.N, d.K, d.b_sn, d.b_sk, d.b_sb, bp, st);
        if (rc) return rc;
    }
    const int bk = d.bk == 16 ? 16 : 32;
    CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
    const int b_rows = d.pair ? 128 : BN;  // a pair CTA holds half of the 256-row B tile
    encode_operand(&m_ahi, ahi, d.M, d.K, ap, bk, BM);
    encode_operand(&m_alo, alo, d.M, d.K, ap, bk, BM);
    encode_operand(&m_bhi, bhi, d.N, d.K, bp, bk, b_rows);
    encode_operand(&m_blo, blo, d.N, d.K, bp, bk, b_rows);
    const int64_t nkb = (d.K + bk - 1) / bk;
    TcParams p;
    p.group_m = 1;
    p.M = static_cast<int>(d.M);
    p.N = static_cast<int>(d.N);
    p.K = static_cast<int>(d.K);
    p.a_batched = d.a_sb != 0;
    p.b_batched = d.b_sb != 0;
    p.ksplit = d.ksplit;
    p.kb_per_split = static_cast<int>((nkb + d.ksplit - 1) / d.ksplit);
    p.chunk_kb = d.chunk_kb > 0 ? d.chunk_kb : 256 / bk;
    p.status = status;
    p.n_full = 0;
    p.tail_split = 0;
    p.tail_kb = 0;
    p.tail_part = nullptr;
    if (d.ksplit > 1) {
        p.C = partial;
        p.ldc = d.N;
        p.c_bstride = d.M * d.N;  // partial index (batch * ksplit + split)
        p.epilogue = EP_NONE;
    } else {
        p.C = C;
        p.ldc = d.N;
        p.c_bstride = d.c_sb;
        p.epilogue = d.epilogue;
    }
    if (d.pair) {
        p.tiles_m = static_cast<int>((d.M + 255) / 256);
        p.tiles_n = static_cast<int>((d.N + 255) / 256);
        p.n_units = static_cast<int>(p.tiles_m * p.tiles_n * d.batch * d.ksplit);
        // Groups of 8 tile rows when rows of tiles are long: at 8192^3 (32 tile columns)
        // the 74 clusters of a wave would otherwise stream 32 B panels and 2-3 A panels at
        // once (measured 263-266 -> 278-282 TFLOP/s with groups).  At 16 tile columns (the
        // MLP's 4096-wide products) groups read 3-11 % fewer DRAM bytes but ran within
        // +-1 % of rows (1 % slower at K = 1024), so rows stay there.
        p.group_m = p.tiles_n > 16 ? TT_GEMM_GROUP_M : 1;
        if (d.tail_split > 0) {
            if (d.ksplit != 1) return static_cast<int>(cudaErrorInvalidValue);  // the planner never does this
            const int T = p.n_units;
            p.n_full = T - d.tail_tiles;
            p.tail_split = d.tail_split;
            p.tail_kb = static_cast<int>((nkb + d.tail_split - 1) / d.tail_split + p.chunk_kb - 1) / p.chunk_kb *
                        p.chunk_kb;
            p.tail_part = partial;
            p.n_units = p.n_full + d.tail_tiles * d.tail_split;
        }
        rc = launch_pair<32>(m_ahi, m_alo, m_bhi, m_blo, p, st);
        if (rc == 0 && d.tail_split > 0) {
            tail_reduce_kernel<<<dim3(16, static_cast<unsigned>(d.tail_tiles)), 256, 0, st>>>(
                partial, C, p.M, p.N, d.N, d.c_sb, p.tiles_m, p.tiles_n, p.group_m, p.n_full, d.tail_split,
                d.epilogue);
            rc = static_cast<int>(cudaGetLastError());
        }
    } else {
        dim3 grid(static_cast<unsigned>((d.N + BN - 1) / BN), static_cast<unsigned>((d.M + BM - 1) / BM),
                  static_cast<unsigned>(d.batch * d.ksplit));
        rc = bk == 16 ? launch_main<16>(m_ahi, m_alo, m_bhi, m_blo, p, grid, st)
                      : launch_main<32>(m_ahi, m_alo, m_bhi, m_blo, p, grid, st);
    }
    if (rc || d.ksplit == 1) return rc;
    return launch_splitk_reduce(partial, C, d.M * d.N, d.ksplit, d.batch, d.c_sb, d.epilogue, st);
}

namespace {
// A barrier that nothing arrives at: the GEMM kernels' bounded wait must give up after
// `budget` cycles, raise the abort flag, record ST_TIMEOUT_FULL in the status word and
// return, leaving the context usable.
__global__ void bounded_wait_selftest_kernel(int* status, long long budget) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, status, ST_TIMEOUT_FULL, budget);
    __syncthreads();
}
}  // namespace

int launch_bounded_wait_selftest(int* status, long long budget, void* stream) {
    bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, budget);
    return static_cast<int>(cudaGetLastError());
}

int launch_splitk_reduce(const float* P, float* C, int64_t per, int ksplit, int64_t batch, int64_t c_sb, int epilogue,
                         void* stream) {
    int64_t blocks = (per + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    splitk_reduce_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(batch)), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(P, C, per, ksplit, c_sb, epilogue);
    return static_cast<int>(cudaGetLastError());
}

int64_t gemm_tc_ctas(const GemmDesc& d) {
    if (d.algo != 2) return 0;
    return ctas_of(d) * d.ksplit + (d.tail_split > 0 ? 2LL * d.tail_tiles * (d.tail_split - 1) : 0);
}

int gemm_tc_launch_count(const GemmDesc& d) {
    int n = 1;
    if (d.M && d.K && !d.a_presplit) ++n;
    if (d.N && d.K && !d.b_presplit) ++n;
    if (d.ksplit > 1 || d.tail_split > 0) ++n;
    return n;
}

}  // namespace ttb
