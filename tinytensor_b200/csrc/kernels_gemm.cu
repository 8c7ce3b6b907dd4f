// GEMM dispatch for C[b] = A[b] . B[b] (float32 in, float32 out).
//
// Two kernels:
//  - gemm_tc:   the tcgen05/TMEM 3xTF32 kernel (kernels_gemm_tc.cu) for shapes whose
//               operands TMA can describe (16-B aligned rows);
//  - gemm_simt: this file's CUDA-core FFMA kernel, used for the small or oddly strided
//               products the tensor-core kernel does not take (e.g. N = 10 outputs).
// Both compute the reference's C = A.B (src/core/operators.cpp:235-319) with fp32
// accumulation; operands may be K-major or M/N-major views (transposes are folded
// into the strides, never materialised).
#include <cuda_runtime.h>

#include <cstdint>

#include "program.hpp"

namespace ttb {

int launch_gemm_tc(const GemmDesc& d, const float* A, const float* B, float* C, void* scratch, int* status,
                   void* stream, const GemmSplitIO* io);
bool gemm_tc_supported(const GemmDesc& d);
int64_t gemm_tc_scratch_bytes(const GemmDesc& d);
int gemm_tc_launch_count(const GemmDesc& d);
void gemm_tc_plan(GemmDesc& d);

namespace {

// 128x128 tile, BK = 8, 256 threads, each thread an 8x8 sub-tile split as rows
// {ty*4..+3, 64+ty*4..+3} x cols {tx*4..+3, 64+tx*4..+3} so shared-memory reads are
// float4 and conflict free.  Double-buffered shared memory.
constexpr int BM = 128, BN = 128, BK = 8;

template <int EPI>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                        float* __restrict__ C, int64_t M, int64_t N, int64_t K,
                                                        int64_t a_sm, int64_t a_sk, int64_t a_sb, int64_t b_sk,
                                                        int64_t b_sn, int64_t b_sb, int64_t c_sb) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    const int64_t bz = blockIdx.z;
    A += bz * a_sb;
    B += bz * b_sb;
    C += bz * c_sb;
    const bool a_kmaj = (a_sk == 1);
    const bool b_nmaj = (b_sn == 1);

    // Each thread loads 4 elements of each tile; the mapping follows the unit stride.
    auto load_tiles = [&](int64_t k0, float ra[4], float rb[4]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = tid * 4 + j;
            int mm, kk;
            if (a_kmaj) { mm = e >> 3; kk = e & 7; } else { kk = e >> 7; mm = e & 127; }
            const int64_t gm = m0 + mm, gk = k0 + kk;
            ra[j] = (gm < M && gk < K) ? __ldg(A + gm * a_sm + gk * a_sk) : 0.0f;
            int nn;
            if (b_nmaj) { kk = e >> 7; nn = e & 127; } else { nn = e >> 3; kk = e & 7; }
            const int64_t gn = n0 + nn, gk2 = k0 + kk;
            rb[j] = (gn < N && gk2 < K) ? __ldg(B + gk2 * b_sk + gn * b_sn) : 0.0f;
        }
    };
    auto store_tiles = [&](int buf, const float ra[4], const float rb[4]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = tid * 4 + j;
            int mm, kk;
            if (a_kmaj) { mm = e >> 3; kk = e & 7; } else { kk = e >> 7; mm = e & 127; }
            As[buf][kk][mm] = ra[j];
            int nn;
            if (b_nmaj) { kk = e >> 7; nn = e & 127; } else { nn = e >> 3; kk = e & 7; }
            Bs[buf][kk][nn] = rb[j];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    float ra[4], rb[4];
    load_tiles(0, ra, rb);
    store_tiles(0, ra, rb);
    __syncthreads();
    int buf = 0;
    for (int64_t k0 = 0; k0 < K; k0 += BK) {
        const bool more = k0 + BK < K;
        if (more) load_tiles(k0 + BK, ra, rb);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[8];
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_tiles(buf ^ 1, ra, rb);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (gn < N) {
                float v = acc[i][j];
                v = gemm_epilogue(v, EPI);
                C[gm * N + gn] = v;
            }
        }
    }
}

// Skinny products: at most 8*G output columns (N <= 16, or M <= 16 with the roles of A
// and B exchanged).  Output (r, q) of batch b is sum_k X[b][r][k] * Y[b][k][q], with
//   X[b][r][k] = X[b*x_sb + r*x_sr + k*x_sk],  Y[b][k][q] = Y[b*y_sb + k*y_sk + q*y_sq],
// stored at C[z*c_sb + r*c_sr + q*c_sq], z = blockIdx.y (batch, or batch*ksplit + split
// when K is split across CTAs and the partials are summed afterwards).
// CTA: 128 rows x all columns over one K range, 128*G threads; thread (g, row) owns
// columns 8g..8g+7 of one row.  X tiles (128 rows x 32 K) are staged transposed,
// Xs[k][row], and double-buffered through registers; XMAJ names the contiguous index of
// X (XM_K: k, XM_R: r, XM_GENERIC: neither) so that global loads are coalesced float4s.
// Sums are kept in 256-K chunks added with RN adds: the rounding error stays that of a
// 256-term sum at any K.  The kernel is bound by reading X once.
enum { XM_GENERIC = 0, XM_K = 1, XM_R = 2 };

template <int G, int XMAJ>
__global__ void __launch_bounds__(128 * G) gemm_skinny_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, float* __restrict__ C, int64_t R, int64_t Q, int64_t K,
    int64_t x_sr, int64_t x_sk, int64_t x_sb, int64_t y_sk, int64_t y_sq, int64_t y_sb, int64_t c_sr, int64_t c_sq,
    int64_t c_sb, int64_t k_per_split, int ksplit, int epilogue) {
    constexpr int TR = 128, TK = 32, NQ = 8 * G, THR = 128 * G;
    constexpr int PAD = XMAJ == XM_R ? 4 : 1;  // XM_R stores float4 rows; others scalar, conflict-free at +1
    constexpr int XV = TR * TK / 4 / THR;      // 4-float groups of the X tile per thread
    constexpr int YV = TK * NQ / THR;          // Y tile elements per thread (2)
    __shared__ __align__(16) float Xs[2][TK][TR + PAD];
    __shared__ __align__(16) float Ys[2][TK][NQ];
    const int tid = threadIdx.x;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * TR;
    const int64_t bz = blockIdx.y / ksplit;
    const int64_t kb = static_cast<int64_t>(blockIdx.y - bz * ksplit) * k_per_split;
    const int64_t ke = K < kb + k_per_split ? K : kb + k_per_split;
    X += bz * x_sb;
    Y += bz * y_sb;
    C += static_cast<int64_t>(blockIdx.y) * c_sb;

    float xr[XV][4], yr[YV];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < XV; ++i) {
            const int e = tid + i * THR;
            if (XMAJ == XM_R) {
                const int64_t k = k0 + e / 32, r = r0 + (e % 32) * 4;
                if (k < ke && r + 3 < R) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(X + k * x_sk + r));
                    xr[i][0] = v.x; xr[i][1] = v.y; xr[i][2] = v.z; xr[i][3] = v.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) xr[i][j] = (k < ke && r + j < R) ? __ldg(X + k * x_sk + r + j) : 0.0f;
                }
            } else {
                const int64_t r = r0 + e / 8, k = k0 + (e % 8) * 4;
                if (XMAJ == XM_K && r < R && k + 3 < ke) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(X + r * x_sr + k));
                    xr[i][0] = v.x; xr[i][1] = v.y; xr[i][2] = v.z; xr[i][3] = v.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        xr[i][j] = (r < R && k + j < ke) ? __ldg(X + r * x_sr + (k + j) * x_sk) : 0.0f;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < YV; ++i) {
            const int e = tid + i * THR;
            const int64_t k = k0 + e / NQ, q = e % NQ;
            yr[i] = (k < ke && q < Q) ? __ldg(Y + k * y_sk + q * y_sq) : 0.0f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < XV; ++i) {
            const int e = tid + i * THR;
            if (XMAJ == XM_R) {
                *reinterpret_cast<float4*>(&Xs[buf][e / 32][(e % 32) * 4]) =
                    make_float4(xr[i][0], xr[i][1], xr[i][2], xr[i][3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) Xs[buf][(e % 8) * 4 + j][e / 8] = xr[i][j];
            }
        }
#pragma unroll
        for (int i = 0; i < YV; ++i) {
            const int e = tid + i * THR;
            Ys[buf][e / NQ][e % NQ] = yr[i];
        }
    };

    const int row = tid & (TR - 1), g = tid / TR;
    float acc[8], tot[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = tot[j] = 0.0f;
    load(kb);
    store(0);
    __syncthreads();
    int buf = 0, tile = 0;
    for (int64_t k0 = kb; k0 < ke; k0 += TK, ++tile) {
        const bool more = k0 + TK < ke;
        if (more) load(k0 + TK);
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            const float a = Xs[buf][kk][row];
            const float4 b0 = *reinterpret_cast<const float4*>(&Ys[buf][kk][g * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Ys[buf][kk][g * 8 + 4]);
            acc[0] = fmaf(a, b0.x, acc[0]);
            acc[1] = fmaf(a, b0.y, acc[1]);
            acc[2] = fmaf(a, b0.z, acc[2]);
            acc[3] = fmaf(a, b0.w, acc[3]);
            acc[4] = fmaf(a, b1.x, acc[4]);
            acc[5] = fmaf(a, b1.y, acc[5]);
            acc[6] = fmaf(a, b1.z, acc[6]);
            acc[7] = fmaf(a, b1.w, acc[7]);
        }
        if ((tile & 7) == 7) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                tot[j] = __fadd_rn(tot[j], acc[j]);
                acc[j] = 0.0f;
            }
        }
        if (more) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    const int64_t r = r0 + row;
    if (r < R) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t q = g * 8 + j;
            if (q < Q) {
                float v = __fadd_rn(tot[j], acc[j]);
                v = gemm_epilogue(v, epilogue);
                C[r * c_sr + q * c_sq] = v;
            }
        }
    }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Skinny products whose X is read in 16-B pieces (XM_K: k contiguous, XM_R: r
// contiguous; 16-B aligned rows).  Same output mapping as gemm_skinny_kernel; here
// X tiles (128 rows x 32 K, 16 KB) stream through a 4-stage cp.async ring straight
// into shared memory (src-size zero-fill at the edges), and one thread owns one row and
// all NQ (4..16, a multiple of 4) columns.  XM_K tiles stay row-major with each row's
// 16-B chunks XOR-swizzled by the row (chunk c of row r at c ^ (r & 7)), so a warp's
// per-row float4 reads are conflict-free; XM_R tiles are stored [k][row].  Sums are kept
// in 256-K chunks added with RN adds, as in gemm_skinny_kernel.
constexpr int SKA_TR = 128, SKA_TK = 32, SKA_ST = 4;

template <int NQ>
constexpr int skinny_async_smem() {
    return SKA_ST * (SKA_TR * SKA_TK + SKA_TK * NQ) * 4;
}

template <int NQ, int XMAJ>
__global__ void __launch_bounds__(128) gemm_skinny_async_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, float* __restrict__ C, int64_t R, int64_t Q, int64_t K,
    int64_t x_sr, int64_t x_sk, int64_t x_sb, int64_t y_sk, int64_t y_sq, int64_t y_sb, int64_t c_sr, int64_t c_sq,
    int64_t c_sb, int64_t k_per_split, int ksplit, int epilogue) {
    constexpr int TR = SKA_TR, TK = SKA_TK, ST = SKA_ST;
    extern __shared__ __align__(16) float ska_smem[];
    float* Xs = ska_smem;                       // [ST][TR * TK]
    float* Ys = ska_smem + ST * TR * TK;        // [ST][TK][NQ]
    const int tid = threadIdx.x;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * TR;
    const int64_t bz = blockIdx.y / ksplit;
    const int64_t kb = static_cast<int64_t>(blockIdx.y - bz * ksplit) * k_per_split;
    const int64_t ke = K < kb + k_per_split ? K : kb + k_per_split;
    X += bz * x_sb;
    Y += bz * y_sb;
    C += static_cast<int64_t>(blockIdx.y) * c_sb;
    const int ntiles = ke > kb ? static_cast<int>((ke - kb + TK - 1) / TK) : 0;

    auto issue = [&](int t) {
        const int s = t % ST;
        const int64_t k0 = kb + static_cast<int64_t>(t) * TK;
        float* xs = Xs + s * TR * TK;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = tid + i * 128;
            int bytes = 0;
            const float* src = X;
            float* dst;
            if (XMAJ == XM_K) {
                const int rr = e >> 3, c = e & 7;
                const int64_t r = r0 + rr, k = k0 + 4 * c;
                if (r < R && k < ke) {
                    bytes = ke - k >= 4 ? 16 : static_cast<int>(4 * (ke - k));
                    src = X + r * x_sr + k;
                }
                dst = xs + rr * TK + ((c ^ (rr & 7)) << 2);
            } else {
                const int kk = e >> 5, c = e & 31;
                const int64_t k = k0 + kk, r = r0 + 4 * c;
                if (k < ke && r < R) {
                    bytes = R - r >= 4 ? 16 : static_cast<int>(4 * (R - r));
                    src = X + k * x_sk + r;
                }
                dst = xs + kk * TR + 4 * c;
            }
            cp_async16(dst, src, bytes);
        }
        float* ys = Ys + s * TK * NQ;
        for (int e = tid; e < TK * NQ; e += 128) {
            const int kk = e / NQ, q = e - kk * NQ;
            const int64_t k = k0 + kk;
            const bool in = k < ke && q < Q;
            cp_async4(ys + e, in ? Y + k * y_sk + q * y_sq : Y, in ? 4 : 0);
        }
    };

    float acc[NQ], tot[NQ];
#pragma unroll
    for (int j = 0; j < NQ; ++j) acc[j] = tot[j] = 0.0f;
#pragma unroll
    for (int t = 0; t < ST - 1; ++t) {
        if (t < ntiles) issue(t);
        cp_async_commit();
    }
    const int rr = tid;
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<ST - 2>();
        __syncthreads();
        if (t + ST - 1 < ntiles) issue(t + ST - 1);
        cp_async_commit();
        const int s = t % ST;
        const float* xs = Xs + s * TR * TK;
        const float* ys = Ys + s * TK * NQ;
        if (XMAJ == XM_K) {
#pragma unroll
            for (int c = 0; c < TK / 4; ++c) {
                const float4 a4 = *reinterpret_cast<const float4*>(xs + rr * TK + ((c ^ (rr & 7)) << 2));
                const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float* yk = ys + (4 * c + j) * NQ;
#pragma unroll
                    for (int q4 = 0; q4 < NQ / 4; ++q4) {
                        const float4 b = *reinterpret_cast<const float4*>(yk + 4 * q4);
                        acc[4 * q4 + 0] = fmaf(av[j], b.x, acc[4 * q4 + 0]);
                        acc[4 * q4 + 1] = fmaf(av[j], b.y, acc[4 * q4 + 1]);
                        acc[4 * q4 + 2] = fmaf(av[j], b.z, acc[4 * q4 + 2]);
                        acc[4 * q4 + 3] = fmaf(av[j], b.w, acc[4 * q4 + 3]);
                    }
                }
            }
        } else {
#pragma unroll 8
            for (int kk = 0; kk < TK; ++kk) {
                const float a = xs[kk * TR + rr];
                const float* yk = ys + kk * NQ;
#pragma unroll
                for (int q4 = 0; q4 < NQ / 4; ++q4) {
                    const float4 b = *reinterpret_cast<const float4*>(yk + 4 * q4);
                    acc[4 * q4 + 0] = fmaf(a, b.x, acc[4 * q4 + 0]);
                    acc[4 * q4 + 1] = fmaf(a, b.y, acc[4 * q4 + 1]);
                    acc[4 * q4 + 2] = fmaf(a, b.z, acc[4 * q4 + 2]);
                    acc[4 * q4 + 3] = fmaf(a, b.w, acc[4 * q4 + 3]);
                }
            }
        }
        if ((t & 7) == 7) {
#pragma unroll
            for (int j = 0; j < NQ; ++j) {
                tot[j] = __fadd_rn(tot[j], acc[j]);
                acc[j] = 0.0f;
            }
        }
    }
    cp_async_wait<0>();
    const int64_t r = r0 + rr;
    if (r < R) {
#pragma unroll
        for (int j = 0; j < NQ; ++j) {
            if (j < Q) {
                float v = __fadd_rn(tot[j], acc[j]);
                v = gemm_epilogue(v, epilogue);
                C[r * c_sr + j * c_sq] = v;
            }
        }
    }
}

// Skinny products with X read along k (x_sk = 1, 16-B aligned rows) and Y a contiguous
// [K][Q] block (16-B aligned), Q <= 16: the output layer Y = H.W of a network.  CTA:
// 256 threads over 8*RW rows and one K range; each stage of a 4-stage cp.async ring
// holds an X tile (8*RW rows x 128 k) and the matching 128 x Q block of Y.  Warp w owns
// rows w, w+8, .. of a tile and lane l the four k's 4l..4l+3, so a warp reads each of
// its rows as one conflict-free 512-B float4 load, and the lane's 4 x Q values of Y
// (4Q consecutive floats: Q float4 loads from shared memory) are loaded once per tile and
// used for all RW rows: per tile a warp issues Q + RW loads for 4*RW*Q FMAs, with no
// padding of Q.  Each lane sums its k's in order (fmaf), the warp then adds the 32
// lanes' sums by a shuffle tree (every lane ends with the same bits), and split partials
// are added in split order by the split-K reduce: deterministic.  A split holds at most
// SK2_MAX_K of K, so a lane's sum has at most SK2_MAX_K / 32 terms.
#ifndef TT_SK2_RW
#define TT_SK2_RW 4
#endif
constexpr int SK2_RW = TT_SK2_RW, SK2_TR = 8 * SK2_RW, SK2_TK = 128, SK2_ST = 4;
constexpr int64_t SK2_MAX_K = 8192;
// Y block per stage: the 32 lanes' groups of 4 k x Q floats (Q 16-B chunks each), each
// group padded to an odd number of chunks so that the lanes' float4 reads of their own
// group hit distinct banks (a stride of an even number of chunks put lanes l and l+4 of
// an 8-lane phase on the same banks: 2.6 M conflicts per launch at 8192 x 10 x 4096).
template <int Q>
constexpr int sk2_group_floats() {
    return 4 * (Q % 2 ? Q : Q + 1);
}
template <int Q>
constexpr int sk2_wfloats() {
    return 32 * sk2_group_floats<Q>();
}
template <int Q>
constexpr int sk2_smem() {
    return SK2_ST * (SK2_TR * SK2_TK + sk2_wfloats<Q>()) * 4;
}

template <int Q>
__global__ void __launch_bounds__(256, SK2_RW <= 4 ? 2 : 1) gemm_skinny_k2_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, float* __restrict__ C, int64_t R, int64_t K,
    int64_t x_sr, int64_t x_sb, int64_t y_sb, int64_t c_sr, int64_t c_sq, int64_t c_sb, int64_t k_per_split,
    int ksplit, int epilogue) {
    constexpr int TR = SK2_TR, TK = SK2_TK, ST = SK2_ST, RW = SK2_RW, WF = sk2_wfloats<Q>();
    constexpr int STAGE = TR * TK + WF;
    extern __shared__ __align__(16) float sk2_smem_buf[];  // [ST][X tile | Y block]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * TR;
    const int64_t bz = blockIdx.y / ksplit;
    const int64_t kb = static_cast<int64_t>(blockIdx.y - bz * ksplit) * k_per_split;
    const int64_t ke = K < kb + k_per_split ? K : kb + k_per_split;
    X += bz * x_sb;
    Y += bz * y_sb;
    C += static_cast<int64_t>(blockIdx.y) * c_sb;
    const int ntiles = ke > kb ? static_cast<int>((ke - kb + TK - 1) / TK) : 0;

    // This thread's copy plan, fixed over the K range: X chunk i of a stage is row
    // tid/32 + 8i of the tile at k's 4(tid%32)..+3, Y chunk j is e = tid + 256j of the
    // block's 32Q chunks.  Interior tiles (all TR rows inside R, all TK k's inside the
    // split) copy by pointer adds alone; edge tiles take the per-chunk checks below.
    constexpr int XCH = TR * TK / 4 / 256, YCH = (32 * Q + 255) / 256;
    const bool rows_full = r0 + TR <= R;
    const float* xrow = rows_full ? X + (r0 + (tid >> 5)) * x_sr + kb + 4 * (tid & 31) : X;
    const int64_t xstep = 8 * x_sr;
    const int xdst = (tid >> 5) * TK + 4 * (tid & 31);
    int ydst[YCH];
#pragma unroll
    for (int j = 0; j < YCH; ++j) {
        const int e = tid + 256 * j, g = e / Q;
        ydst[j] = g * sk2_group_floats<Q>() + 4 * (e - g * Q);
    }

    auto issue = [&](int t) {
        float* xs = sk2_smem_buf + (t % ST) * STAGE;
        const int64_t k0 = kb + static_cast<int64_t>(t) * TK;
        if (rows_full && k0 + TK <= ke) {
            const float* xp = xrow + static_cast<int64_t>(t) * TK;
#pragma unroll
            for (int i = 0; i < XCH; ++i) cp_async16(xs + xdst + 8 * i * TK, xp + i * xstep, 16);
            const float* yp = Y + k0 * Q;
#pragma unroll
            for (int j = 0; j < YCH; ++j)
                if (tid + 256 * j < 32 * Q) cp_async16(xs + TR * TK + ydst[j], yp + 4 * (tid + 256 * j), 16);
            return;
        }
#pragma unroll
        for (int i = 0; i < XCH; ++i) {
            const int e = tid + i * 256;
            const int rr = e >> 5, c = e & 31;
            const int64_t r = r0 + rr, k = k0 + 4 * c;
            int bytes = 0;
            const float* src = X;
            if (r < R && k < ke) {
                bytes = ke - k >= 4 ? 16 : static_cast<int>(4 * (ke - k));
                src = X + r * x_sr + k;
            }
            cp_async16(xs + rr * TK + 4 * c, src, bytes);
        }
        // Y rows k0 .. k0+127: 128*Q consecutive floats (zero past the K range), chunk e
        // to lane group e / Q at its padded place
        float* ws = xs + TR * TK;
        const int64_t wlim = (ke - k0) * Q;  // floats of this block inside the K range
        for (int e = tid; e < 32 * Q; e += 256) {
            const int64_t f = 4 * static_cast<int64_t>(e);
            const int g = e / Q, c = e - g * Q;
            const int bytes = f >= wlim ? 0 : (wlim - f >= 4 ? 16 : static_cast<int>(4 * (wlim - f)));
            cp_async16(ws + g * sk2_group_floats<Q>() + 4 * c, bytes ? Y + k0 * Q + f : Y, bytes);
        }
    };

    float acc[RW][Q];
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
        for (int q = 0; q < Q; ++q) acc[i][q] = 0.0f;
#pragma unroll
    for (int t = 0; t < ST - 1; ++t) {
        if (t < ntiles) issue(t);
        cp_async_commit();
    }
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<ST - 2>();
        __syncthreads();
        if (t + ST - 1 < ntiles) issue(t + ST - 1);
        cp_async_commit();
        const float* xs = sk2_smem_buf + (t % ST) * STAGE;
        // this lane's 4 k's of Y: its group (4Q floats of the block, at the padded place)
        const float4* w4 = reinterpret_cast<const float4*>(xs + TR * TK + lane * sk2_group_floats<Q>());
        float w[4 * Q];
#pragma unroll
        for (int v = 0; v < Q; ++v) {
            const float4 f = w4[v];
            w[4 * v] = f.x;
            w[4 * v + 1] = f.y;
            w[4 * v + 2] = f.z;
            w[4 * v + 3] = f.w;
        }
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            const float4 x = *reinterpret_cast<const float4*>(xs + (warp + 8 * i) * TK + 4 * lane);
#pragma unroll
            for (int q = 0; q < Q; ++q) {
                float a = acc[i][q];
                a = fmaf(x.x, w[q], a);
                a = fmaf(x.y, w[Q + q], a);
                a = fmaf(x.z, w[2 * Q + q], a);
                a = fmaf(x.w, w[3 * Q + q], a);
                acc[i][q] = a;
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int i = 0; i < RW; ++i) {
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            float v = acc[i][q];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const int64_t r = r0 + warp + 8 * i;
            if (lane == (i * Q + q) % 32 && r < R) C[r * c_sr + q * c_sq] = gemm_epilogue(v, epilogue);
        }
    }
}

// Skinny products with X read along r (x_sr = 1, x_sk % 4 == 0, 16-B aligned): the
// weight gradient dW = H^T.dY of an output layer, H row-major.  CTA: 256 threads over
// 256 r and one K range; X tiles (32 k x 256 r, 32 KB) and Y tiles (32 k x Q, padded to
// QP) stream through a 3-stage cp.async ring.  Warp w owns r-half w & 1 (128 r, lane l
// the 4 r's 4l..4l+3) and the k's kk = w >> 1 (mod 4) of a tile: per k one conflict-free
// float4 load of X, QP/4 broadcast float4 loads of Y and 4Q FMAs.  Each lane sums its
// k's in order, the four k-groups' sums are then added in group order through shared
// memory, and split partials in split order: deterministic.  A split holds at most
// SR2_MAX_K of K (a lane's sum has at most SR2_MAX_K / 4 terms).
constexpr int SR2_TR = 256, SR2_TK = 32, SR2_ST = 3;
constexpr int64_t SR2_MAX_K = 2048;

template <int Q>
constexpr int sr2_qp() {
    return (Q + 3) / 4 * 4;
}
template <int Q>
constexpr int sr2_smem() {
    return SR2_ST * (SR2_TK * SR2_TR + SR2_TK * sr2_qp<Q>()) * 4;
}

template <int Q>
__global__ void __launch_bounds__(256, 2) gemm_skinny_r2_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, float* __restrict__ C, int64_t R, int64_t K,
    int64_t x_sk, int64_t x_sb, int64_t y_sk, int64_t y_sq, int64_t y_sb, int64_t c_sr, int64_t c_sq, int64_t c_sb,
    int64_t k_per_split, int ksplit, int epilogue) {
    constexpr int TR = SR2_TR, TK = SR2_TK, ST = SR2_ST, QP = sr2_qp<Q>();
    extern __shared__ __align__(16) float sr2_smem[];
    float* Xs = sr2_smem;                 // [ST][TK][TR]
    float* Ys = sr2_smem + ST * TK * TR;  // [ST][TK][QP]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rh = warp & 1, kg = warp >> 1;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * TR;
    const int64_t bz = blockIdx.y / ksplit;
    const int64_t kb = static_cast<int64_t>(blockIdx.y - bz * ksplit) * k_per_split;
    const int64_t ke = K < kb + k_per_split ? K : kb + k_per_split;
    X += bz * x_sb;
    Y += bz * y_sb;
    C += static_cast<int64_t>(blockIdx.y) * c_sb;
    const int ntiles = ke > kb ? static_cast<int>((ke - kb + TK - 1) / TK) : 0;

    // This thread's copy plan, fixed over the K range: X chunk i of a stage is k row
    // tid/64 + 4i of the tile at r's 4(tid%64)..+3, Y element j is e = tid + 256j of the
    // TK x QP block.  Interior tiles (all TR r's inside R, all TK k's inside the split)
    // copy by pointer adds alone; edge tiles take the per-chunk checks below.
    constexpr int XCH = TK * TR / 4 / 256, YCH = (TK * QP + 255) / 256;
    const bool rows_full = r0 + TR <= R;
    const float* xcol = rows_full ? X + (kb + (tid >> 6)) * x_sk + r0 + 4 * (tid & 63) : X;
    const int64_t xstep = 4 * x_sk;
    const int xdst = (tid >> 6) * TR + 4 * (tid & 63);
    int64_t yoff[YCH];
    bool yin[YCH];
#pragma unroll
    for (int j = 0; j < YCH; ++j) {
        const int e = tid + 256 * j, kk = e / QP, q = e - kk * QP;
        yin[j] = e < TK * QP && q < Q;
        yoff[j] = kk * y_sk + q * y_sq;
    }

    auto issue = [&](int t) {
        const int s = t % ST;
        float* xs = Xs + s * TK * TR;
        const int64_t k0 = kb + static_cast<int64_t>(t) * TK;
        if (rows_full && k0 + TK <= ke) {
            const float* xp = xcol + static_cast<int64_t>(t) * TK * x_sk;
#pragma unroll
            for (int i = 0; i < XCH; ++i) cp_async16(xs + xdst + 4 * i * TR, xp + i * xstep, 16);
            float* ys = Ys + s * TK * QP;
            const float* yp = Y + k0 * y_sk;
#pragma unroll
            for (int j = 0; j < YCH; ++j)
                if (tid + 256 * j < TK * QP) cp_async4(ys + tid + 256 * j, yin[j] ? yp + yoff[j] : Y, yin[j] ? 4 : 0);
            return;
        }
#pragma unroll
        for (int i = 0; i < XCH; ++i) {
            const int e = tid + i * 256;
            const int kk = e >> 6, c = e & 63;
            const int64_t k = k0 + kk, r = r0 + 4 * c;
            int bytes = 0;
            const float* src = X;
            if (k < ke && r < R) {
                bytes = R - r >= 4 ? 16 : static_cast<int>(4 * (R - r));
                src = X + k * x_sk + r;
            }
            cp_async16(xs + kk * TR + 4 * c, src, bytes);
        }
        float* ys = Ys + s * TK * QP;
        for (int e = tid; e < TK * QP; e += 256) {
            const int kk = e / QP, q = e - kk * QP;
            const int64_t k = k0 + kk;
            const bool in = k < ke && q < Q;
            cp_async4(ys + e, in ? Y + k * y_sk + q * y_sq : Y, in ? 4 : 0);
        }
    };

    float acc[4][Q];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int q = 0; q < Q; ++q) acc[j][q] = 0.0f;
#pragma unroll
    for (int t = 0; t < ST - 1; ++t) {
        if (t < ntiles) issue(t);
        cp_async_commit();
    }
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<ST - 2>();
        __syncthreads();
        if (t + ST - 1 < ntiles) issue(t + ST - 1);
        cp_async_commit();
        const int s = t % ST;
        const float* xs = Xs + s * TK * TR + rh * 128 + 4 * lane;
        const float* ys = Ys + s * TK * QP;
#pragma unroll 4
        for (int kk = kg; kk < TK; kk += 4) {
            const float4 x = *reinterpret_cast<const float4*>(xs + kk * TR);
            const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int q4 = 0; q4 < QP / 4; ++q4) {
                const float4 y = *reinterpret_cast<const float4*>(ys + kk * QP + 4 * q4);
                const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (4 * q4 + u < Q) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[j][4 * q4 + u] = fmaf(xv[j], yv[u], acc[j][4 * q4 + u]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    // k-groups 1..3 park their sums; group 0 adds them in group order and stores
    float* red = sr2_smem;  // [3][2][32][4][Q] floats, inside the ring
    if (kg > 0) {
        float* d = red + ((((kg - 1) * 2 + rh) * 32 + lane) * 4) * Q;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < Q; ++q) d[j * Q + q] = acc[j][q];
    }
    __syncthreads();
    if (kg == 0) {
#pragma unroll
        for (int g = 0; g < 3; ++g) {
            const float* d = red + (((g * 2 + rh) * 32 + lane) * 4) * Q;
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int q = 0; q < Q; ++q) acc[j][q] = __fadd_rn(acc[j][q], d[j * Q + q]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t r = r0 + rh * 128 + 4 * lane + j;
            if (r < R) {
#pragma unroll
                for (int q = 0; q < Q; ++q) C[r * c_sr + q * c_sq] = gemm_epilogue(acc[j][q], epilogue);
            }
        }
    }
}

// Products with K <= 16 (bound by writing C).  A CTA owns one 128-column strip of C:
// it stages B (K x 128) in shared memory once and keeps each thread's 4 columns of it
// in registers (KP <= 16 float4s, K padded with zeros), then walks row blocks of 64
// (blockIdx.y, grid-stride), double-buffering the A block (64 x K) through registers.
// Thread (ty, tx) computes rows ty + 8i (i < 8) x columns 4tx..4tx+3 (float4 stores when
// C's rows allow it).  Each output is one sequential fmaf sum over k < K (the zero
// padding adds exact zeros).
template <int KP, int EPI>
__global__ void __launch_bounds__(256) gemm_smallk_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                          float* __restrict__ C, int64_t M, int64_t N, int K,
                                                          int64_t a_sm, int64_t a_sk, int64_t a_sb, int64_t b_sk,
                                                          int64_t b_sn, int64_t b_sb, int64_t c_sb, int vec_store) {
    __shared__ __align__(16) float As[2][64][16];
    __shared__ __align__(16) float Bs[16][128];
    const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 128;
    const int64_t bz = blockIdx.z;
    A += bz * a_sb;
    B += bz * b_sb;
    C += bz * c_sb;
    for (int e = tid; e < KP * 128; e += 256) {
        const int k = e >> 7, nn = e & 127;
        Bs[k][nn] = (k < K && n0 + nn < N) ? __ldg(B + k * b_sk + (n0 + nn) * b_sn) : 0.0f;
    }
    const int64_t row_tiles = (M + 63) / 64;
    float ar[4];
    auto load_a = [&](int64_t mt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = tid + 256 * j, rr = e >> 4, k = e & 15;
            const int64_t m = mt * 64 + rr;
            ar[j] = (m < M && k < K) ? __ldg(A + m * a_sm + k * a_sk) : 0.0f;
        }
    };
    auto store_a = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = tid + 256 * j;
            As[buf][e >> 4][e & 15] = ar[j];
        }
    };
    int64_t mt = blockIdx.y;
    if (mt < row_tiles) {
        load_a(mt);
        store_a(0);
    }
    __syncthreads();
    float4 bk[KP];
#pragma unroll
    for (int k = 0; k < KP; ++k) bk[k] = *reinterpret_cast<const float4*>(&Bs[k][4 * tx]);
    const int64_t n = n0 + 4 * tx;
    int buf = 0;
    for (; mt < row_tiles; mt += gridDim.y) {
        const int64_t next = mt + gridDim.y;
        if (next < row_tiles) load_a(next);
#pragma unroll 2
        for (int i = 0; i < 8; ++i) {
            const int rr = ty + 8 * i;
            const int64_t m = mt * 64 + rr;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k4 = 0; k4 < KP / 4; ++k4) {
                const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][rr][4 * k4]);
                const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 b = bk[4 * k4 + j];
                    v[0] = fmaf(av[j], b.x, v[0]);
                    v[1] = fmaf(av[j], b.y, v[1]);
                    v[2] = fmaf(av[j], b.z, v[2]);
                    v[3] = fmaf(av[j], b.w, v[3]);
                }
            }
            if (EPI != EP_NONE) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = gemm_epilogue(v[j], EPI);
            }
            if (m >= M) continue;
            float* crow = C + m * N;
            if (vec_store && n + 3 < N) {
                *reinterpret_cast<float4*>(crow + n) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (n + j < N) crow[n + j] = v[j];
            }
        }
        if (next < row_tiles) store_a(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
}

// One wave: a CTA per 128-column strip and row-block walker, as many as fit on the GPU.
template <int KP>
void launch_smallk_t(const GemmDesc& d, const float* A, const float* B, float* C, int vec, cudaStream_t st) {
    static const int per_sm = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemm_smallk_kernel<KP, EP_NONE>, 256, 0) != cudaSuccess)
            n = 2;
        return n > 0 ? n : 1;
    }();
    const int64_t col_tiles = (d.N + 127) / 128, row_tiles = (d.M + 63) / 64;
    int64_t walkers = (148 * per_sm + col_tiles * d.batch - 1) / (col_tiles * d.batch);
    if (walkers > row_tiles) walkers = row_tiles;
    if (walkers > 65535) walkers = 65535;
    if (walkers < 1) walkers = 1;
    dim3 grid(static_cast<unsigned>(col_tiles), static_cast<unsigned>(walkers), static_cast<unsigned>(d.batch));
    const int K = static_cast<int>(d.K);
    if (d.epilogue == EP_RELU)
        gemm_smallk_kernel<KP, EP_RELU><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, K, d.a_sm, d.a_sk, d.a_sb, d.b_sk,
                                                              d.b_sn, d.b_sb, d.c_sb, vec);
    else if (d.epilogue == EP_TANH)
        gemm_smallk_kernel<KP, EP_TANH><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, K, d.a_sm, d.a_sk, d.a_sb, d.b_sk,
                                                              d.b_sn, d.b_sb, d.c_sb, vec);
    else
        gemm_smallk_kernel<KP, EP_NONE><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, K, d.a_sm, d.a_sk, d.a_sb, d.b_sk,
                                                              d.b_sn, d.b_sb, d.c_sb, vec);
}

enum Algo { ALGO_SIMT = 0, ALGO_SKINNY = 1, ALGO_TC = 2, ALGO_SKINNY_T = 3, ALGO_SMALLK = 4 };

// Operand roles of the skinny kernel: X has the long rows, Y the <= 16 columns.
struct SkinnyView {
    int64_t R, Q;
    const float* X;
    const float* Y;
    int64_t x_sr, x_sk, x_sb, y_sk, y_sq, y_sb, c_sr, c_sq;
};

SkinnyView skinny_view(const GemmDesc& d, const float* A, const float* B) {
    SkinnyView v;
    if (d.algo == ALGO_SKINNY_T) {  // C^T = B^T . A^T: rows along N, columns along M
        v = {d.N, d.M, B, A, d.b_sn, d.b_sk, d.b_sb, d.a_sk, d.a_sm, d.a_sb, 1, d.N};
    } else {
        v = {d.M, d.N, A, B, d.a_sm, d.a_sk, d.a_sb, d.b_sk, d.b_sn, d.b_sb, d.N, 1};
    }
    return v;
}

int64_t skinny_k_per_split(const GemmDesc& d) {
    const int64_t per = (d.K + d.ksplit - 1) / d.ksplit;
    return (per + 31) / 32 * 32;
}

template <int G, int XMAJ>
void launch_skinny_t(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, dim3 grid, cudaStream_t st) {
    gemm_skinny_kernel<G, XMAJ><<<grid, 128 * G, 0, st>>>(v.X, v.Y, out, v.R, v.Q, d.K, v.x_sr, v.x_sk, v.x_sb, v.y_sk,
                                                         v.y_sq, v.y_sb, v.c_sr, v.c_sq, out_sb, skinny_k_per_split(d),
                                                         d.ksplit, d.ksplit > 1 ? EP_NONE : d.epilogue);
}

template <int NQ, int XMAJ>
void launch_skinny_async_t(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, dim3 grid,
                           cudaStream_t st) {
    static bool attr = [] {
        return cudaFuncSetAttribute(gemm_skinny_async_kernel<NQ, XMAJ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    skinny_async_smem<NQ>()) == cudaSuccess;
    }();
    (void)attr;
    gemm_skinny_async_kernel<NQ, XMAJ><<<grid, 128, skinny_async_smem<NQ>(), st>>>(
        v.X, v.Y, out, v.R, v.Q, d.K, v.x_sr, v.x_sk, v.x_sb, v.y_sk, v.y_sq, v.y_sb, v.c_sr, v.c_sq, out_sb,
        skinny_k_per_split(d), d.ksplit, d.ksplit > 1 ? EP_NONE : d.epilogue);
}

template <int XMAJ>
void launch_skinny_async(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, dim3 grid,
                         cudaStream_t st) {
    if (v.Q <= 4) launch_skinny_async_t<4, XMAJ>(v, d, out, out_sb, grid, st);
    else if (v.Q <= 8) launch_skinny_async_t<8, XMAJ>(v, d, out, out_sb, grid, st);
    else if (v.Q <= 12) launch_skinny_async_t<12, XMAJ>(v, d, out, out_sb, grid, st);
    else launch_skinny_async_t<16, XMAJ>(v, d, out, out_sb, grid, st);
}

// Which skinny kernel a view's strides select (alignment is checked again at launch).
enum SkinnyKind { SK_OLD = 0, SK_K2 = 1, SK_R2 = 2 };
SkinnyKind skinny_kind(const SkinnyView& v) {
    if (v.Q > 16) return SK_OLD;
    if (v.x_sk == 1 && v.x_sr % 4 == 0 && v.y_sq == 1 && v.y_sk == v.Q) return SK_K2;
    if (v.x_sr == 1 && v.x_sk % 4 == 0) return SK_R2;
    return SK_OLD;
}

template <int Q>
void launch_k2_t(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, cudaStream_t st) {
    static bool attr = [] {
        return cudaFuncSetAttribute(gemm_skinny_k2_kernel<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    sk2_smem<Q>()) == cudaSuccess;
    }();
    (void)attr;
    dim3 grid(static_cast<unsigned>((v.R + SK2_TR - 1) / SK2_TR), static_cast<unsigned>(d.batch * d.ksplit));
    gemm_skinny_k2_kernel<Q><<<grid, 256, sk2_smem<Q>(), st>>>(v.X, v.Y, out, v.R, d.K, v.x_sr, v.x_sb, v.y_sb, v.c_sr,
                                                         v.c_sq, out_sb, skinny_k_per_split(d), d.ksplit,
                                                         d.ksplit > 1 ? EP_NONE : d.epilogue);
}

template <int Q>
void launch_r2_t(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, cudaStream_t st) {
    static bool attr = [] {
        return cudaFuncSetAttribute(gemm_skinny_r2_kernel<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    sr2_smem<Q>()) == cudaSuccess;
    }();
    (void)attr;
    dim3 grid(static_cast<unsigned>((v.R + SR2_TR - 1) / SR2_TR), static_cast<unsigned>(d.batch * d.ksplit));
    gemm_skinny_r2_kernel<Q><<<grid, 256, sr2_smem<Q>(), st>>>(v.X, v.Y, out, v.R, d.K, v.x_sk, v.x_sb, v.y_sk, v.y_sq,
                                                              v.y_sb, v.c_sr, v.c_sq, out_sb, skinny_k_per_split(d),
                                                              d.ksplit, d.ksplit > 1 ? EP_NONE : d.epilogue);
}

#define TT_SKINNY_Q_CASES(F) \
    F(1) F(2) F(3) F(4) F(5) F(6) F(7) F(8) F(9) F(10) F(11) F(12) F(13) F(14) F(15) F(16)

void launch_k2(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, cudaStream_t st) {
    switch (v.Q) {
#define TT_K2_CASE(q) \
    case q: launch_k2_t<q>(v, d, out, out_sb, st); break;
        TT_SKINNY_Q_CASES(TT_K2_CASE)
#undef TT_K2_CASE
        default: break;
    }
}

void launch_r2(const SkinnyView& v, const GemmDesc& d, float* out, int64_t out_sb, cudaStream_t st) {
    switch (v.Q) {
#define TT_R2_CASE(q) \
    case q: launch_r2_t<q>(v, d, out, out_sb, st); break;
        TT_SKINNY_Q_CASES(TT_R2_CASE)
#undef TT_R2_CASE
        default: break;
    }
}

int launch_skinny(const GemmDesc& d, const float* A, const float* B, float* C, void* scratch, cudaStream_t st) {
    const SkinnyView v = skinny_view(d, A, B);
    const bool x16 = (reinterpret_cast<uintptr_t>(v.X) & 15) == 0 && (d.batch == 1 || v.x_sb % 4 == 0);
    const bool y16 = (reinterpret_cast<uintptr_t>(v.Y) & 15) == 0 && (d.batch == 1 || v.y_sb % 4 == 0);
    float* out = d.ksplit > 1 ? static_cast<float*>(scratch) : C;
    const int64_t out_sb = d.ksplit > 1 ? d.M * d.N : d.c_sb;
    dim3 grid(static_cast<unsigned>((v.R + 127) / 128), static_cast<unsigned>(d.batch * d.ksplit));
    const SkinnyKind kind = skinny_kind(v);
    if (x16 && y16 && kind == SK_K2) {
        launch_k2(v, d, out, out_sb, st);
    } else if (x16 && kind == SK_R2) {
        launch_r2(v, d, out, out_sb, st);
    } else if (x16 && v.x_sk == 1 && v.x_sr % 4 == 0) {
        launch_skinny_async<XM_K>(v, d, out, out_sb, grid, st);
    } else if (x16 && v.x_sr == 1 && v.x_sk % 4 == 0) {
        launch_skinny_async<XM_R>(v, d, out, out_sb, grid, st);
    } else if (v.Q > 8) {
        launch_skinny_t<2, XM_GENERIC>(v, d, out, out_sb, grid, st);
    } else {
        launch_skinny_t<1, XM_GENERIC>(v, d, out, out_sb, grid, st);
    }
    int rc = static_cast<int>(cudaGetLastError());
    if (rc || d.ksplit == 1) return rc;
    return launch_splitk_reduce(out, C, d.M * d.N, d.ksplit, d.batch, d.c_sb, d.epilogue, st);
}

// Split-K of the skinny kernels.  K2 / R2 (one / two resident CTAs per SM): a wave model
// like the tensor-core planner's — waves x (tiles per split + a ramp of ~2 tiles) plus
// the partials' extra HBM traffic in tile times — under the kernels' cap on K per split.
// Others: enough CTAs for ~2 waves of 3 per SM, each split >= 256 of K.
int64_t plan_skinny_split(int64_t ctas, int64_t K, int64_t tk, int64_t max_k, int64_t slots, double tile_bytes_hbm,
                          double out_bytes, int64_t batch) {
    const int64_t ntk = (K + tk - 1) / tk;
    const int64_t smin = (K + max_k - 1) / max_k;
    int64_t best = smin;
    double best_cost = -1.0;
    for (int64_t ks = smin; ks <= smin + 256 && ks <= ntk && ks * batch <= 65535; ++ks) {
        const int64_t per = (ntk + ks - 1) / ks;
        const int64_t waves = (ctas * ks + slots - 1) / slots;
        double cost = static_cast<double>(waves) * (static_cast<double>(per) + 2.0);
        if (ks > 1) cost += 2.0 * static_cast<double>(ks) * out_bytes / tile_bytes_hbm;
        if (best_cost < 0.0 || cost < best_cost) {
            best_cost = cost;
            best = ks;
        }
    }
    return best;
}

void plan_skinny(GemmDesc& d) {
    const int64_t R = d.algo == ALGO_SKINNY_T ? d.N : d.M;
    const SkinnyView v = skinny_view(d, nullptr, nullptr);
    const double out_bytes = static_cast<double>(d.M) * static_cast<double>(d.N) * 4.0 * static_cast<double>(d.batch);
    // HBM bytes moved (whole GPU) while one CTA streams one tile: 32 KB tiles at the
    // per-SM share of ~6.5 TB/s, shared by the CTAs resident on the SM
    const SkinnyKind kind = skinny_kind(v);
    if (kind == SK_K2) {
        const int64_t per_sm = SK2_RW <= 4 ? 2 : 1;
        const double tile_bytes = static_cast<double>(SK2_TR * SK2_TK * 4);
        d.ksplit = static_cast<int>(plan_skinny_split((R + SK2_TR - 1) / SK2_TR * d.batch, d.K, SK2_TK, SK2_MAX_K,
                                                      148 * per_sm, 148.0 * static_cast<double>(per_sm) * tile_bytes,
                                                      out_bytes, d.batch));
        return;
    }
    if (kind == SK_R2) {
        d.ksplit = static_cast<int>(plan_skinny_split((R + SR2_TR - 1) / SR2_TR * d.batch, d.K, SR2_TK, SR2_MAX_K,
                                                      296, 2.0 * 148.0 * 32768.0, out_bytes, d.batch));
        return;
    }
    const int64_t ctas = (R + 127) / 128 * d.batch;
    int64_t ks = 1;
    if (ctas < 148 * 6) {
        ks = (148 * 6 + ctas - 1) / ctas;
        const int64_t cap = (d.K + 255) / 256;
        if (ks > cap) ks = cap;
        if (ks * d.batch > 65535) ks = 65535 / d.batch;
        if (ks < 1) ks = 1;
    }
    d.ksplit = static_cast<int>(ks);
}

}  // namespace

void plan_gemm(GemmDesc& d) {
    // Size-1 dims: their stride is never used; make it unit so the layout test passes.
    if (d.M == 1) d.a_sm = 1;
    if (d.K == 1) {
        d.a_sk = 1;
        d.b_sk = 1;
    }
    if (d.N == 1) d.b_sn = 1;
    d.ksplit = 1;
    const bool batch_ok = d.batch <= 65535;
    if (batch_ok && d.K <= 16 && (d.N + 127) / 128 <= 65535) {
        d.algo = ALGO_SMALLK;
    } else if (batch_ok && d.N <= 16) {
        d.algo = ALGO_SKINNY;
        plan_skinny(d);
    } else if (batch_ok && d.M <= 16) {
        d.algo = ALGO_SKINNY_T;
        plan_skinny(d);
    } else if (gemm_tc_supported(d)) {
        d.algo = ALGO_TC;
        gemm_tc_plan(d);
    } else {
        d.algo = ALGO_SIMT;
    }
}

const char* gemm_algo_name(int algo) {
    switch (algo) {
        case ALGO_TC: return "tcgen05_3xtf32";
        case ALGO_SKINNY: return "simt_skinny";
        case ALGO_SKINNY_T: return "simt_skinny_t";
        case ALGO_SMALLK: return "simt_smallk";
        default: return "simt";
    }
}

int64_t gemm_scratch_bytes(const GemmDesc& d) {
    if (d.algo == ALGO_TC) return gemm_tc_scratch_bytes(d);
    if ((d.algo == ALGO_SKINNY || d.algo == ALGO_SKINNY_T) && d.ksplit > 1) return d.batch * d.ksplit * d.M * d.N * 4;
    return 0;
}

int gemm_launch_count(const GemmDesc& d) {
    if (d.M == 0 || d.N == 0 || d.batch == 0) return 0;
    if (d.K == 0) return static_cast<int>(d.batch);
    if (d.algo == ALGO_TC) return gemm_tc_launch_count(d);
    if (d.algo == ALGO_SKINNY || d.algo == ALGO_SKINNY_T) return d.ksplit > 1 ? 2 : 1;
    return 1;
}

int launch_gemm(const GemmDesc& d, const float* A, const float* B, float* C, void* scratch, int* status,
                void* stream, const GemmSplitIO* io) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (d.M == 0 || d.N == 0 || d.batch == 0) return 0;
    A += d.a_off;
    B += d.b_off;
    if (d.K == 0) {
        // C = 0 (operators.cpp:256-259 returns zeros)
        for (int64_t b = 0; b < d.batch; ++b) {
            int rc = launch_fill_f32(C + b * d.c_sb, d.M * d.N, 0.0f, stream);
            if (rc) return rc;
        }
        return 0;
    }
    if (d.algo == ALGO_TC) return launch_gemm_tc(d, A, B, C, scratch, status, stream, io);
    if (d.algo == ALGO_SKINNY || d.algo == ALGO_SKINNY_T) return launch_skinny(d, A, B, C, scratch, st);
    if (d.algo == ALGO_SMALLK) {
        const int vec = d.N % 4 == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0 && d.c_sb % 4 == 0;
        if (d.K <= 4) launch_smallk_t<4>(d, A, B, C, vec, st);
        else if (d.K <= 8) launch_smallk_t<8>(d, A, B, C, vec, st);
        else if (d.K <= 12) launch_smallk_t<12>(d, A, B, C, vec, st);
        else launch_smallk_t<16>(d, A, B, C, vec, st);
        return static_cast<int>(cudaGetLastError());
    }
    dim3 grid(static_cast<unsigned>((d.N + BN - 1) / BN), static_cast<unsigned>((d.M + BM - 1) / BM),
              static_cast<unsigned>(d.batch));
    if (d.epilogue == EP_RELU)
        gemm_simt_kernel<EP_RELU><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, d.K, d.a_sm, d.a_sk, d.a_sb, d.b_sk, d.b_sn,
                                                        d.b_sb, d.c_sb);
    else if (d.epilogue == EP_TANH)
        gemm_simt_kernel<EP_TANH><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, d.K, d.a_sm, d.a_sk, d.a_sb, d.b_sk, d.b_sn,
                                                        d.b_sb, d.c_sb);
    else
        gemm_simt_kernel<EP_NONE><<<grid, 256, 0, st>>>(A, B, C, d.M, d.N, d.K, d.a_sm, d.a_sk, d.a_sb, d.b_sk, d.b_sn,
                                                        d.b_sb, d.c_sb);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace ttb
