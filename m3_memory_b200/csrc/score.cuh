// score.cuh -- the reference's distance in its exact arithmetic, plus the error
// bounds that let a faster approximate score stand in for it during selection.
#pragma once

#include "common.cuh"

namespace m3g {

// unified_score of AgentMemory/M3/include/base.h:22-31 with the kernels of
// AgentMemory/M3/src/base.cpp:12-41, evaluated with the reference's own
// rounding: fp32, one rounding per multiply / add / subtract (the reference is
// built for baseline x86-64, which has no FMA), summed in index order.  The
// explicit _rn intrinsics keep nvcc from contracting into FMAs.  `a` is read
// with stride 1 from any memory space; `b` likewise.
__device__ __forceinline__ float exact_score(const float* __restrict__ a,
                                             const float* __restrict__ b, int d, int metric,
                                             bool normalized) {
    if (metric == kL2) {
        float s = 0.f;
        for (int i = 0; i < d; ++i) {
            float df = __fsub_rn(a[i], b[i]);
            s = __fadd_rn(s, __fmul_rn(df, df));
        }
        return s;
    }
    if (metric == kIP || normalized) {
        float s = 0.f;
        for (int i = 0; i < d; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
        return metric == kIP ? -s : __fsub_rn(1.f, s);
    }
    float dot = 0.f, na = 0.f, nb = 0.f;
    for (int i = 0; i < d; ++i) {
        dot = __fadd_rn(dot, __fmul_rn(a[i], b[i]));
        na = __fadd_rn(na, __fmul_rn(a[i], a[i]));
        nb = __fadd_rn(nb, __fmul_rn(b[i], b[i]));
    }
    if (na == 0.f || nb == 0.f) return 1.f;
    return __fsub_rn(1.f, __fdiv_rn(dot, __fsqrt_rn(__fmul_rn(na, nb))));
}

// Bounds for selecting by an approximate inner product.
//
// `dot` approximates <q, c> with |dot - <q,c>| <= beta * nq * nc, where nq, nc
// are upper bounds of the Euclidean norms.  gamma bounds the reference's own
// sequential-sum error relative to the same norm product (D * 2^-24, with slack).
// On return [lo, hi] contains both the exact real-valued unified score and the
// reference's rounded one, for every metric.  qn2 / cn2 are the squared norms in
// fp32 (used only by L2's approximate value).  Zero-norm vectors under
// non-normalised COSINE make the interval unbounded: the reference special-cases
// them (base.cpp:39) and the exact recheck must decide.
__device__ __forceinline__ void approx_bounds(float dot, float nq, float nc, float qn2, float cn2,
                                              float beta, float gamma, int metric,
                                              bool normalized, float* lo, float* hi,
                                              float* approx = nullptr) {
    const float INF = __int_as_float(0x7f800000);
    float a, e;
    // beta, gamma already carry 1% slack; the factor 1.01 below covers the fp32
    // roundings of this bound's own arithmetic (relative 1e-7 each).
    if (metric == kL2) {
        a = qn2 + cn2 - 2.f * dot;
        float s = nq + nc;
        // 2|dot err| <= beta (nq+nc)^2 / 2; reference error <= gamma (nq+nc)^2;
        // the three-term fp32 sum and the squared norms: <= 8 u (nq+nc)^2
        e = (beta + gamma + 4.8e-7f) * (s * s) * 1.01f;
    } else if (metric == kIP) {
        a = -dot;
        e = (beta + gamma) * (nq * nc) * 1.01f;
    } else if (normalized) {
        a = 1.f - dot;
        e = (beta + gamma) * (nq * nc) * 1.01f + 2.4e-7f * (fabsf(a) + 1.f);
    } else {
        float den = nq * nc;
        if (!(nq > 1e-15f && nc > 1e-15f && nq < 1e15f && nc < 1e15f)) {
            *lo = -INF;
            *hi = INF;
            if (approx) *approx = 0.f;
            return;
        }
        a = 1.f - dot / den;
        e = (beta + 2.f * gamma) * 1.01f + 1e-6f + 2.4e-7f * (fabsf(a) + 1.f);
    }
    e = e + 1e-30f;
    if (approx) *approx = a;
    if (!(fabsf(a) < INF) || !(e < INF)) {
        *lo = -INF;
        *hi = INF;
        return;
    }
    *lo = __fsub_rd(a, e);
    *hi = __fadd_ru(a, e);
}

// The same exact score computed by one warp: the per-element products (each
// rounded, as the reference's a[i] * b[i]) in parallel, then lane 0 adds them
// in index order.  `prod` is a per-warp shared buffer of 3 * chunk floats.
// All lanes return the score.
__device__ __forceinline__ float warp_exact_score(const float* __restrict__ a,
                                                  const float* __restrict__ b, int d, int metric,
                                                  bool normalized, float* prod, int chunk,
                                                  int lane) {
    const bool cos_raw = metric == kCosine && !normalized;
    float s = 0.f, na = 0.f, nb = 0.f;
    for (int d0 = 0; d0 < d; d0 += chunk) {
        const int n = min(chunk, d - d0);
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            const float x = a[d0 + i], y = b[d0 + i];
            if (metric == kL2) {
                const float df = __fsub_rn(x, y);
                prod[i] = __fmul_rn(df, df);
            } else {
                prod[i] = __fmul_rn(x, y);
                if (cos_raw) {
                    prod[chunk + i] = __fmul_rn(x, x);
                    prod[2 * chunk + i] = __fmul_rn(y, y);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            const int n4 = n & ~3;
            if (cos_raw) {
                for (int i = 0; i < n4; i += 4) {
                    const float4 p = *reinterpret_cast<const float4*>(prod + i);
                    const float4 pa = *reinterpret_cast<const float4*>(prod + chunk + i);
                    const float4 pb = *reinterpret_cast<const float4*>(prod + 2 * chunk + i);
                    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, p.x), p.y), p.z), p.w);
                    na = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(na, pa.x), pa.y), pa.z), pa.w);
                    nb = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(nb, pb.x), pb.y), pb.z), pb.w);
                }
                for (int i = n4; i < n; ++i) {
                    s = __fadd_rn(s, prod[i]);
                    na = __fadd_rn(na, prod[chunk + i]);
                    nb = __fadd_rn(nb, prod[2 * chunk + i]);
                }
            } else {
#pragma unroll 4
                for (int i = 0; i < n4; i += 4) {
                    const float4 p = *reinterpret_cast<const float4*>(prod + i);
                    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, p.x), p.y), p.z), p.w);
                }
                for (int i = n4; i < n; ++i) s = __fadd_rn(s, prod[i]);
            }
        }
    }
    float r;
    if (metric == kL2) r = s;
    else if (metric == kIP) r = -s;
    else if (normalized) r = __fsub_rn(1.f, s);
    else r = (na == 0.f || nb == 0.f) ? 1.f : __fsub_rn(1.f, __fdiv_rn(s, __fsqrt_rn(__fmul_rn(na, nb))));
    return __shfl_sync(0xffffffffu, r, 0);
}

// VW consecutive floats from p (global memory) into x; p is 4*VW-byte aligned.
template <int VW>
__device__ __forceinline__ void load_vec(const float* __restrict__ p, float (&x)[VW]) {
    if constexpr (VW == 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else if constexpr (VW == 2) {
        const float2 v = __ldg(reinterpret_cast<const float2*>(p));
        x[0] = v.x; x[1] = v.y;
    } else {
        x[0] = __ldg(p);
    }
}

// VW consecutive floats of x to p (shared memory), p 4*VW-byte aligned.
template <int VW>
__device__ __forceinline__ void store_vec(float* p, const float (&x)[VW]) {
    if constexpr (VW == 4) *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    else if constexpr (VW == 2) *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    else p[0] = x[0];
}

// Row stride (floats) of the product tile of warp_exact_scores<VW>: a chunk of
// 32*VW products plus 4 floats of padding, so that the 128-bit reads of eight
// lanes on eight different rows hit disjoint banks.
template <int VW>
__host__ __device__ constexpr int exact_tile_stride() { return 32 * VW + 4; }
// Floats of the per-warp product tile, enough for every VW in {1, 2, 4}.
constexpr int kExactTileFloats = 32 * (32 + 4);

// The exact score for up to G = 32 / VW candidates at once, one per lane
// (lanes 0 .. G-1): the warp computes the per-element products of a chunk of
// 32 * VW dims for every candidate (each rounded, as the reference's
// a[i] * b[i]) into a shared tile, then each candidate's lane adds its row in
// index order, which is the reference's summation order.  The next chunk's
// centroid values are loaded before that serial sum, whose 32 * VW dependent
// adds hide the load latency; fewer candidates per warp therefore use wider
// chunks.  `q` is in shared memory, 16-byte aligned, with round_up(d, 4)
// floats; `cid` is the lane's centroid row (-1: none; every lane >= G passes
// -1); `stage` holds kExactTileFloats floats, 16-byte aligned.  All 32 lanes
// call it.  Returns the lane's score (undefined where cid < 0).
template <int VW>
__device__ __forceinline__ float warp_exact_scores(const float* __restrict__ q,
                                                   const float* __restrict__ C, int64_t ldc,
                                                   int d, int metric, bool normalized, int cid,
                                                   float* stage, int lane) {
    constexpr int W = 32 * VW, GM = 32 / VW, RS = exact_tile_stride<VW>();
    static_assert(GM * RS <= kExactTileFloats, "tile too small");
    const bool cos_raw = metric == kCosine && !normalized;
    const bool vec = (ldc % VW) == 0 && (reinterpret_cast<uintptr_t>(C) % (4 * VW)) == 0;
    float x[GM][VW];
    auto load = [&](int d0) {
        const int dd = d0 + lane * VW;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            const int cc = __shfl_sync(0xffffffffu, cid, g);
            if (cc >= 0 && vec && dd + VW <= d) {
                load_vec<VW>(C + (int64_t)cc * ldc + dd, x[g]);
            } else {
#pragma unroll
                for (int v = 0; v < VW; ++v)
                    x[g][v] = (cc >= 0 && dd + v < d) ? __ldg(C + (int64_t)cc * ldc + dd + v) : 0.f;
            }
        }
    };
    const bool mine = lane < GM && cid >= 0;
    const float* row = stage + lane * RS;
    float s = 0.f, na = 0.f, nb = 0.f;
    load(0);
    for (int d0 = 0; d0 < d; d0 += W) {
        const int dd = d0 + lane * VW;
        const int nn = min(W, d - d0);
        float qv[VW];
#pragma unroll
        for (int v = 0; v < VW; ++v) qv[v] = dd + v < d ? q[dd + v] : 0.f;
        __syncwarp();  // the previous chunk's sums are done with the tile
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            float p[VW];
#pragma unroll
            for (int v = 0; v < VW; ++v) {
                if (metric == kL2) {
                    const float df = __fsub_rn(qv[v], x[g][v]);
                    p[v] = __fmul_rn(df, df);
                } else {
                    p[v] = __fmul_rn(qv[v], x[g][v]);
                }
            }
            store_vec<VW>(stage + g * RS + lane * VW, p);
        }
        if (!cos_raw && d0 + W < d) load(d0 + W);  // x is free once the products are stored
        __syncwarp();
        if (mine) {
            if (nn == W) {
#pragma unroll
                for (int l = 0; l < W; l += 4) {
                    const float4 r = *reinterpret_cast<const float4*>(row + l);
                    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, r.x), r.y), r.z), r.w);
                }
            } else {
                for (int l = 0; l < nn; ++l) s = __fadd_rn(s, row[l]);
            }
        }
        if (cos_raw) {
            __syncwarp();
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                float p[VW];
#pragma unroll
                for (int v = 0; v < VW; ++v) p[v] = __fmul_rn(x[g][v], x[g][v]);
                store_vec<VW>(stage + g * RS + lane * VW, p);
            }
            if (d0 + W < d) load(d0 + W);
            __syncwarp();
            if (mine) {
                for (int l = 0; l < nn; ++l) {
                    nb = __fadd_rn(nb, row[l]);
                    const float a = q[d0 + l];
                    na = __fadd_rn(na, __fmul_rn(a, a));
                }
            }
        }
    }
    __syncwarp();
    if (metric == kL2) return s;
    if (metric == kIP) return -s;
    if (normalized) return __fsub_rn(1.f, s);
    return (na == 0.f || nb == 0.f) ? 1.f
                                    : __fsub_rn(1.f, __fdiv_rn(s, __fsqrt_rn(__fmul_rn(na, nb))));
}

}  // namespace m3g
