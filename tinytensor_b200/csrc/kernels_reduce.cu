// Sum / mean / max reductions for sm_100a.
//
// Semantics restate the reference's eager ops (src/core/operators.cpp:394-516):
// float32 data accumulated in double, cast to float at the end; mean is
// float(sum) * float(1/count) in float.  max (no reference op) keeps a float
// running maximum with IEEE 754-2019 maximum() semantics (NaN propagates, -0 < +0),
// so the result is order independent and bit-exact against the CPU oracle.
//
// Layouts (views folded by the scheduler, so a transposed input costs nothing):
//   ROW  out[o] = red_r x[o*s_outer + r]     one warp per (row, split); float4 when possible
//   COL  out[o] = red_r x[r*s_red + o]       one thread per (4 columns, split); float4
//   GEN  any strides                          one thread per output
// With splits > 1 each (row|column, split) writes a double partial to scratch and a
// finishing kernel combines the partials in a fixed order (deterministic).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "program.hpp"

namespace ttb {

namespace {

constexpr int kThreads = 256;

template <int OP>
struct Acc;
template <>
struct Acc<RO_SUM> {
    double v = 0.0;
    __device__ void add(float x) { v += static_cast<double>(x); }
    __device__ void merge(double o) { v += o; }
    __device__ double get() const { return v; }
};
template <>
struct Acc<RO_MEAN> : Acc<RO_SUM> {};
template <>
struct Acc<RO_MAX> {
    float v = -INFINITY;
    // x wins when larger, when NaN, or when both are zeros and v is -0 (x is then +0 or -0)
    __device__ void add(float x) { v = (x > v || x != x || (x == v && __float_as_uint(v) == 0x80000000u)) ? x : v; }
    __device__ void merge(double o) { add(static_cast<float>(o)); }
    __device__ double get() const { return static_cast<double>(v); }
};

template <int OP>
__device__ __forceinline__ float finish(double acc, float scale) {
    float f = static_cast<float>(acc);
    return OP == RO_MEAN ? f * scale : f;
}

template <int OP>
__device__ __forceinline__ double warp_merge(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        double w = __shfl_xor_sync(0xffffffffu, v, o);
        if (OP == RO_MAX) {
            float a = static_cast<float>(v), b = static_cast<float>(w);
            v = (b > a || b != b || (b == a && __float_as_uint(a) == 0x80000000u)) ? w : v;
        } else {
            v += w;
        }
    }
    return v;
}

// ROW: one warp per (row, split).  VEC=4 requires R % 4 == 0 and 16-B aligned rows.
template <int OP, int VEC>
__global__ void __launch_bounds__(kThreads) reduce_row_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                               double* __restrict__ part, int64_t outer, int64_t R,
                                                               int64_t s_outer, int splits, float scale) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= outer * splits) return;
    const int64_t row = warp / splits;
    const int split = static_cast<int>(warp % splits);
    const int64_t nvec = R / VEC;
    const int64_t per = (nvec + splits - 1) / splits;
    const int64_t v0 = per * split;
    const int64_t v1 = v0 + per < nvec ? v0 + per : nvec;
    const float* rp = x + row * s_outer;
    Acc<OP> acc;
    if (VEC == 4) {
        const float4* r4 = reinterpret_cast<const float4*>(rp);
        int64_t v = v0 + lane;
        for (; v + 96 < v1; v += 128) {
            float4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = __ldg(r4 + v + 32 * u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc.add(q[u].x);
                acc.add(q[u].y);
                acc.add(q[u].z);
                acc.add(q[u].w);
            }
        }
        for (; v < v1; v += 32) {
            float4 q = __ldg(r4 + v);
            acc.add(q.x);
            acc.add(q.y);
            acc.add(q.z);
            acc.add(q.w);
        }
    } else {
        for (int64_t v = v0 + lane; v < v1; v += 32) acc.add(__ldg(rp + v));
    }
    double r = warp_merge<OP>(acc.get());
    if (lane == 0) {
        if (splits == 1) out[row] = finish<OP>(r, scale);
        else part[row * splits + split] = r;
    }
}

// ROW with long rows (R >= kCtaRowMin, float4, no split): one CTA per row.  The 8 warps
// read consecutive 4 KB pieces of one row and the CTAs are dispatched in row order, so
// the CTAs resident at one time stream one contiguous window of X, 16 KB runs side by
// side.  (A warp per row puts a stream on every row at once, 8192 streams 16 KB apart
// for [8192, 4096], which costs HBM row-buffer locality: 0.80 of the copy bandwidth
// against 0.90 here.  A persistent-CTA variant streaming 16 KB chunks through a cp.async
// ring ran at 0.81 at best.)  Registers stay at 32 so that 8 CTAs fit per SM: a second
// accumulator chain per thread (40 registers, 6 CTAs per SM) cost 10 %.
// Per-thread partials are merged by a warp shuffle tree, then the 8 warp results in warp
// order: a fixed order, so the result is deterministic.
// max takes the hardware's NaN-propagating maximum (max.NaN.f32, one instruction per
// element).  Its choice between -0 and +0 is not relied on: a row whose maximum is a
// zero is scanned again for a +0 (IEEE 754-2019 maximum: -0 < +0).
constexpr int64_t kCtaRowMin = 2048;

__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

template <int OP>
struct RowAcc : Acc<OP> {};
template <>
struct RowAcc<RO_MAX> {
    float v = -INFINITY;
    __device__ void add(float x) { v = max_nan(v, x); }
    __device__ double get() const { return static_cast<double>(v); }
};

template <int OP>
__global__ void __launch_bounds__(kThreads, 8) reduce_row_cta_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                                   int64_t R, int64_t s_outer, float scale) {
    __shared__ double wpart[kThreads / 32];
    const int64_t row = blockIdx.x;
    const float4* r4 = reinterpret_cast<const float4*>(x + row * s_outer);
    const int nvec = static_cast<int>(R / 4);
    RowAcc<OP> acc;
    int v = threadIdx.x;
    for (; v + 3 * kThreads < nvec; v += 4 * kThreads) {
        float4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = __ldg(r4 + v + u * kThreads);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            acc.add(q[u].x);
            acc.add(q[u].y);
            acc.add(q[u].z);
            acc.add(q[u].w);
        }
    }
    for (; v < nvec; v += kThreads) {
        const float4 q = __ldg(r4 + v);
        acc.add(q.x);
        acc.add(q.y);
        acc.add(q.z);
        acc.add(q.w);
    }
    double r;
    if (OP == RO_MAX) {
        float m = static_cast<float>(acc.get());
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
        r = static_cast<double>(m);
    } else {
        r = warp_merge<OP>(acc.get());
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wpart[warp] = r;
    __syncthreads();
    if (OP == RO_MAX) {
        float m = -INFINITY;
        for (int w = 0; w < kThreads / 32; ++w) m = max_nan(m, static_cast<float>(wpart[w]));
        if (m == 0.0f) {  // -0 or +0: +0 if the row holds a +0 (all threads agree on m)
            int plus = 0;
            for (int i = threadIdx.x; i < nvec; i += kThreads) {
                const float4 q = __ldg(r4 + i);
                plus |= (__float_as_uint(q.x) == 0u) | (__float_as_uint(q.y) == 0u) | (__float_as_uint(q.z) == 0u) |
                        (__float_as_uint(q.w) == 0u);
            }
            m = __syncthreads_or(plus) ? 0.0f : -0.0f;
        }
        if (threadIdx.x == 0) out[row] = m;
    } else if (threadIdx.x == 0) {
        Acc<OP> t;
        for (int w = 0; w < kThreads / 32; ++w) t.merge(wpart[w]);
        out[row] = finish<OP>(t.get(), scale);
    }
}

// COL: one thread per VEC consecutive columns and one split of the rows.
template <int OP, int VEC>
__global__ void __launch_bounds__(kThreads) reduce_col_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                               double* __restrict__ part, int64_t outer, int64_t R,
                                                               int64_t s_red, int splits, float scale) {
    const int64_t cv = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;  // column vector index
    const int split = blockIdx.y;
    if (cv * VEC >= outer) return;
    const int64_t per = (R + splits - 1) / splits;
    const int64_t r0 = per * split;
    const int64_t r1 = r0 + per < R ? r0 + per : R;
    Acc<OP> acc[VEC];
    if (VEC == 4) {
        const float* base = x + cv * 4;
        int64_t r = r0;
        for (; r + 3 < r1; r += 4) {
            float4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = __ldg(reinterpret_cast<const float4*>(base + (r + u) * s_red));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc[0].add(q[u].x);
                acc[1].add(q[u].y);
                acc[2].add(q[u].z);
                acc[3].add(q[u].w);
            }
        }
        for (; r < r1; ++r) {
            float4 q = __ldg(reinterpret_cast<const float4*>(base + r * s_red));
            acc[0].add(q.x);
            acc[1].add(q.y);
            acc[2].add(q.z);
            acc[3].add(q.w);
        }
    } else {
        for (int64_t r = r0; r < r1; ++r) acc[0].add(__ldg(x + r * s_red + cv));
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        const int64_t o = cv * VEC + k;
        if (splits == 1) out[o] = finish<OP>(acc[k].get(), scale);
        else part[static_cast<int64_t>(split) * outer + o] = acc[k].get();
    }
}

// Combines split partials in split order.  row_major: part[o*splits + s], else part[s*outer + o].
template <int OP>
__global__ void __launch_bounds__(kThreads) reduce_finish_kernel(const double* __restrict__ part,
                                                                  float* __restrict__ out, int64_t outer, int splits,
                                                                  int row_major, float scale) {
    const int64_t o = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (o >= outer) return;
    Acc<OP> acc;
    for (int s = 0; s < splits; ++s) acc.merge(row_major ? part[o * splits + s] : part[static_cast<int64_t>(s) * outer + o]);
    out[o] = finish<OP>(acc.get(), scale);
}

struct GenDims {
    int nk, nr;
    int64_t ksize[TT_MAX_RANK], kstride[TT_MAX_RANK], rsize[TT_MAX_RANK], rstride[TT_MAX_RANK];
};

// GENERIC: one thread per output, reduced elements walked in row-major order.
template <int OP>
__global__ void __launch_bounds__(kThreads) reduce_generic_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                                   int64_t outer, int64_t R, GenDims g, float scale) {
    const int64_t o = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (o >= outer) return;
    int64_t base = 0, t = o;
    for (int d = g.nk - 1; d >= 0; --d) {
        base += (t % g.ksize[d]) * g.kstride[d];
        t /= g.ksize[d];
    }
    Acc<OP> acc;
    for (int64_t r = 0; r < R; ++r) {
        int64_t off = base, u = r;
        for (int d = g.nr - 1; d >= 0; --d) {
            off += (u % g.rsize[d]) * g.rstride[d];
            u /= g.rsize[d];
        }
        acc.add(__ldg(x + off));
    }
    out[o] = finish<OP>(acc.get(), scale);
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
    int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (i < n) p[i] = v;
}

constexpr int64_t kTargetWarps = 148 * 64;

int row_splits(int64_t outer, int64_t R) {
    if (outer <= 0 || outer >= kTargetWarps / 2) return 1;
    int64_t s = (kTargetWarps + outer - 1) / outer;
    int64_t maxs = R / 1024;  // keep >= 1024 elements per warp
    if (s > maxs) s = maxs;
    if (s < 1) s = 1;
    if (s > 4096) s = 4096;
    return static_cast<int>(s);
}

int col_splits(int64_t outer, int64_t R, int vec) {
    if (outer <= 0) return 1;
    int64_t threads = (outer + vec - 1) / vec;
    int64_t target = 148 * 2048;
    if (threads >= target / 2) return 1;
    int64_t s = (target + threads - 1) / threads;
    int64_t maxs = R / 64;
    if (s > maxs) s = maxs;
    if (s < 1) s = 1;
    if (s > 65535) s = 65535;
    return static_cast<int>(s);
}

template <int OP>
int launch_op(const ReduceDesc& d, const float* in, float* out, void* scratch, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    double* part = static_cast<double*>(scratch);
    const float* x = in + d.in_offset;
    if (d.outer == 0) return 0;
    if (d.R == 0) {
        float v = OP == RO_MAX ? -INFINITY : 0.0f;
        fill_kernel<<<static_cast<unsigned>((d.outer + kThreads - 1) / kThreads), kThreads, 0, st>>>(out, d.outer, v);
        return static_cast<int>(cudaGetLastError());
    }
    if (d.kind == RK_ROW && d.vec == 4 && d.splits == 1 && d.R >= kCtaRowMin) {
        reduce_row_cta_kernel<OP><<<static_cast<unsigned>(d.outer), kThreads, 0, st>>>(x, out, d.R, d.s_outer,
                                                                                      d.mean_scale);
    } else if (d.kind == RK_ROW) {
        int64_t warps = d.outer * d.splits;
        unsigned blocks = static_cast<unsigned>((warps * 32 + kThreads - 1) / kThreads);
        if (d.vec == 4)
            reduce_row_kernel<OP, 4><<<blocks, kThreads, 0, st>>>(x, out, part, d.outer, d.R, d.s_outer, d.splits,
                                                                  d.mean_scale);
        else
            reduce_row_kernel<OP, 1><<<blocks, kThreads, 0, st>>>(x, out, part, d.outer, d.R, d.s_outer, d.splits,
                                                                  d.mean_scale);
        if (d.splits > 1)
            reduce_finish_kernel<OP><<<static_cast<unsigned>((d.outer + kThreads - 1) / kThreads), kThreads, 0, st>>>(
                part, out, d.outer, d.splits, 1, d.mean_scale);
    } else if (d.kind == RK_COL) {
        int64_t cvs = (d.outer + d.vec - 1) / d.vec;
        dim3 grid(static_cast<unsigned>((cvs + kThreads - 1) / kThreads), static_cast<unsigned>(d.splits));
        if (d.vec == 4)
            reduce_col_kernel<OP, 4><<<grid, kThreads, 0, st>>>(x, out, part, d.outer, d.R, d.s_red, d.splits,
                                                                d.mean_scale);
        else
            reduce_col_kernel<OP, 1><<<grid, kThreads, 0, st>>>(x, out, part, d.outer, d.R, d.s_red, d.splits,
                                                                d.mean_scale);
        if (d.splits > 1)
            reduce_finish_kernel<OP><<<static_cast<unsigned>((d.outer + kThreads - 1) / kThreads), kThreads, 0, st>>>(
                part, out, d.outer, d.splits, 0, d.mean_scale);
    } else {
        GenDims g;
        g.nk = d.nk;
        g.nr = d.nr;
        for (int k = 0; k < TT_MAX_RANK; ++k) {
            g.ksize[k] = d.ksize[k];
            g.kstride[k] = d.kstride[k];
            g.rsize[k] = d.rsize[k];
            g.rstride[k] = d.rstride[k];
        }
        reduce_generic_kernel<OP><<<static_cast<unsigned>((d.outer + kThreads - 1) / kThreads), kThreads, 0, st>>>(
            x, out, d.outer, d.R, g, d.mean_scale);
    }
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

// Fixes splits / vector width for a descriptor (called once at compile time).
static void finalize_desc(ReduceDesc& d) {
    if (d.kind == RK_ROW) {
        d.vec = (d.R % 4 == 0 && d.s_outer % 4 == 0 && d.in_offset % 4 == 0) ? 4 : 1;
        d.splits = row_splits(d.outer, d.R);
    } else if (d.kind == RK_COL) {
        d.vec = (d.outer % 4 == 0 && d.s_red % 4 == 0 && d.in_offset % 4 == 0) ? 4 : 1;
        d.splits = col_splits(d.outer, d.R, d.vec);
    } else {
        d.splits = 1;
        d.vec = 1;
    }
}

int64_t reduce_prepare(ReduceDesc& d) {
    finalize_desc(d);
    if (d.R == 0 || d.splits <= 1) return 0;
    return d.outer * d.splits * static_cast<int64_t>(sizeof(double));
}

int launch_reduce(const ReduceDesc& d, const float* in, float* out, void* scratch, void* stream) {
    switch (d.op) {
        case RO_SUM: return launch_op<RO_SUM>(d, in, out, scratch, stream);
        case RO_MEAN: return launch_op<RO_MEAN>(d, in, out, scratch, stream);
        default: return launch_op<RO_MAX>(d, in, out, scratch, stream);
    }
}

int launch_fill_f32(float* p, int64_t n, float v, void* stream) {
    if (n <= 0) return 0;
    fill_kernel<<<static_cast<unsigned>((n + kThreads - 1) / kThreads), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        p, n, v);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace ttb
