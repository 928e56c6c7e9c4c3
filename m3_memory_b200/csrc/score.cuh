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

// The exact score for up to 32 candidates at once, one per lane: the warp
// computes the per-element products of 32 dims for all 32 candidates (each
// rounded, as the reference's a[i] * b[i]) into a padded 32 x 33 shared tile,
// then every lane adds its own candidate's row in index order.  `cid` is the
// lane's centroid row (-1: none); `stage` is a per-warp buffer of 32 * 33 floats.
// The next chunk's centroid values are loaded while the current one is summed.
// Returns the lane's score (undefined for cid < 0).
__device__ __forceinline__ float warp_exact_scores32(const float* __restrict__ q,
                                                     const float* __restrict__ C, int64_t ldc,
                                                     int d, int metric, bool normalized, int cid,
                                                     float* stage, int lane) {
    const bool cos_raw = metric == kCosine && !normalized;
    float s = 0.f, na = 0.f, nb = 0.f;
    float xs[32];
    auto load_chunk = [&](int d0, float (&x)[32]) {
        const int dd = d0 + lane;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
            const int cc = __shfl_sync(0xffffffffu, cid, c);
            x[c] = (cc >= 0 && dd < d) ? C[(int64_t)cc * ldc + dd] : 0.f;
        }
    };
    load_chunk(0, xs);
    for (int d0 = 0; d0 < d; d0 += 32) {
        const int dd = d0 + lane;
        const float qv = dd < d ? q[dd] : 0.f;
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
            float p;
            if (metric == kL2) {
                const float df = __fsub_rn(qv, xs[c]);
                p = __fmul_rn(df, df);
            } else {
                p = __fmul_rn(qv, xs[c]);
            }
            stage[c * 33 + lane] = p;
        }
        float xn[32];
        if (cos_raw) {
            __syncwarp();
            const int nn = min(32, d - d0);
            for (int l = 0; l < nn; ++l) s = __fadd_rn(s, stage[lane * 33 + l]);
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 32; ++c) stage[c * 33 + lane] = __fmul_rn(xs[c], xs[c]);
            __syncwarp();
            for (int l = 0; l < nn; ++l) {
                nb = __fadd_rn(nb, stage[lane * 33 + l]);
                const float a = q[d0 + l];
                na = __fadd_rn(na, __fmul_rn(a, a));
            }
            if (d0 + 32 < d) load_chunk(d0 + 32, xn);
        } else {
            if (d0 + 32 < d) load_chunk(d0 + 32, xn);
            __syncwarp();
            const int nn = min(32, d - d0);
            const float* row = stage + lane * 33;
            if (nn == 32) {
#pragma unroll
                for (int l = 0; l < 32; ++l) s = __fadd_rn(s, row[l]);
            } else {
                for (int l = 0; l < nn; ++l) s = __fadd_rn(s, row[l]);
            }
        }
        if (d0 + 32 < d) {
#pragma unroll
            for (int c = 0; c < 32; ++c) xs[c] = xn[c];
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
