// topk.cuh -- warp-level top-k of the list scans: a warp holds one query's best
// keys, key = (score key << 32) | row, ascending, ~0 marking an empty slot;
// rows that beat the current k-th key are buffered in shared memory and merged
// in by a bitonic sort + merge.  RegTopK: k <= 32, lane i holds entry i.
// RegTopKW<KW>: k <= 32 KW, lane i holds entries i, 32 + i, ..., 32 (KW-1) + i.
#pragma once

#include "common.cuh"

namespace m3g {

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
    return ((unsigned long long)hi << 32) | lo;
}

__device__ __forceinline__ unsigned long long shfl_u64(unsigned long long v, int src) {
    const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
    const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
    return ((unsigned long long)hi << 32) | lo;
}

// Bitonic sort of one key per lane, ascending across lanes.
__device__ __forceinline__ unsigned long long warp_sort_asc(unsigned long long v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const unsigned long long p = shfl_xor_u64(v, j);
            const bool up = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            v = (lower == up) ? (p < v ? p : v) : (p > v ? p : v);
        }
    }
    return v;
}

// top (ascending, lane i = entry i) <- the 32 smallest of top and cand (any order).
__device__ __forceinline__ unsigned long long warp_merge_top(unsigned long long top,
                                                             unsigned long long cand, int lane) {
    const unsigned long long b = warp_sort_asc(cand, lane);
    const unsigned long long rb = shfl_u64(b, 31 - lane);
    unsigned long long c = top < rb ? top : rb;  // bitonic: the 32 smallest of both
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const unsigned long long p = shfl_xor_u64(c, j);
        const bool lower = (lane & j) == 0;
        c = lower ? (p < c ? p : c) : (p > c ? p : c);
    }
    return c;
}

// Register top-k (k <= 32) fed through a 32-slot shared-memory buffer: a row
// that beats the current k-th key is appended; the buffer is merged into the
// top list (sort + bitonic merge) only when it would overflow, and once more at
// the end of the item, so merges are rare after the first few rows.
//
// `cap` bounds tau from above: keys at or above it can be left out (a bound
// known from outside this list, see the tensor-core scan's per-query bound).
struct RegTopK {
    unsigned long long top = ~0ull;  // lane i: i-th best key (ascending)
    unsigned long long tau = ~0ull;  // keys below it enter the buffer (all lanes)
    unsigned long long cap = ~0ull;  // upper bound of tau
    int nbuf = 0;                    // keys waiting in the buffer (warp-uniform)

    __device__ __forceinline__ void set_cap(unsigned long long c) {
        cap = c;
        tau = tau < c ? tau : c;
    }

    __device__ __forceinline__ void flush(unsigned long long* buf, int k, int lane) {
        __syncwarp();
        const unsigned long long b = lane < nbuf ? buf[lane] : ~0ull;
        __syncwarp();
        top = warp_merge_top(top, b, lane);
        if (lane >= k) top = ~0ull;
        tau = shfl_u64(top, k - 1);
        tau = tau < cap ? tau : cap;
        nbuf = 0;
    }

    __device__ __forceinline__ void push(unsigned long long* buf, int k, float s, int32_t row,
                                         int lane) {
        const unsigned long long key =
            score_valid(s) ? (((unsigned long long)float_key(s) << 32) | (uint32_t)row) : ~0ull;
        bool cand = key < tau;
        unsigned ball = __ballot_sync(0xffffffffu, cand);
        if (!ball) return;
        int cnt = __popc(ball);
        if (nbuf + cnt > 32) {
            flush(buf, k, lane);
            cand = key < tau;
            ball = __ballot_sync(0xffffffffu, cand);
            cnt = __popc(ball);
        }
        if (cand) buf[nbuf + __popc(ball & ((1u << lane) - 1u))] = key;
        nbuf += cnt;
    }
};

// Second half of a bitonic merge: v is bitonic across the warp; afterwards it
// is ascending.
__device__ __forceinline__ unsigned long long warp_bitonic_clean(unsigned long long v, int lane) {
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const unsigned long long p = shfl_xor_u64(v, j);
        const bool lower = (lane & j) == 0;
        v = lower ? (p < v ? p : v) : (p > v ? p : v);
    }
    return v;
}

// Register top-k of up to 32 KW entries, fed like RegTopK.  A flush sorts the
// buffer and merges it level by level: level w keeps the 32 smallest of its
// entries and the carried keys, and carries the 32 largest on (the smallest 32
// of the union of an ascending list and anything can only come from the
// list's first 32 entries and that thing, so the cascade keeps the whole list
// sorted).  KW = 1 is RegTopK exactly.
template <int KW>
struct RegTopKW {
    unsigned long long top[KW];      // lane i: entries i + 32 w (ascending)
    unsigned long long tau = ~0ull;  // keys below it enter the buffer (all lanes)
    unsigned long long cap = ~0ull;  // upper bound of tau
    int nbuf = 0;                    // keys waiting in the buffer (warp-uniform)

    __device__ __forceinline__ RegTopKW() {
#pragma unroll
        for (int w = 0; w < KW; ++w) top[w] = ~0ull;
    }

    __device__ __forceinline__ void set_cap(unsigned long long c) {
        cap = c;
        tau = tau < c ? tau : c;
    }

    // key of entry e (warp-uniform e < 32 KW), in every lane.  Every level is
    // shuffled and the right one selected, so top[] is never indexed by a runtime
    // value (which would move it to local memory).
    __device__ __forceinline__ unsigned long long entry(int e) const {
        unsigned long long v = ~0ull;
#pragma unroll
        for (int w = 0; w < KW; ++w) {
            const unsigned long long t = shfl_u64(top[w], e & 31);
            v = (e >> 5) == w ? t : v;
        }
        return v;
    }

    __device__ __forceinline__ void flush(unsigned long long* buf, int k, int lane) {
        __syncwarp();
        const unsigned long long b = lane < nbuf ? buf[lane] : ~0ull;
        __syncwarp();
        unsigned long long c = warp_sort_asc(b, lane);
#pragma unroll
        for (int w = 0; w < KW; ++w) {
            const unsigned long long rc = shfl_u64(c, 31 - lane);
            const unsigned long long lo = top[w] < rc ? top[w] : rc;
            const unsigned long long hi = top[w] < rc ? rc : top[w];
            top[w] = warp_bitonic_clean(lo, lane);
            if (w + 1 < KW) {
                // nothing carried on: the lower levels are unchanged
                if (__all_sync(0xffffffffu, hi == ~0ull)) break;
                c = warp_bitonic_clean(hi, lane);
            }
        }
#pragma unroll
        for (int w = 0; w < KW; ++w)
            if (32 * w + lane >= k) top[w] = ~0ull;
        tau = entry(k - 1);
        tau = tau < cap ? tau : cap;
        nbuf = 0;
    }

    __device__ __forceinline__ void push(unsigned long long* buf, int k, float s, int32_t row,
                                         int lane) {
        const unsigned long long key =
            score_valid(s) ? (((unsigned long long)float_key(s) << 32) | (uint32_t)row) : ~0ull;
        bool cand = key < tau;
        unsigned ball = __ballot_sync(0xffffffffu, cand);
        if (!ball) return;
        int cnt = __popc(ball);
        if (nbuf + cnt > 32) {
            flush(buf, k, lane);
            cand = key < tau;
            ball = __ballot_sync(0xffffffffu, cand);
            cnt = __popc(ball);
        }
        if (cand) buf[nbuf + __popc(ball & ((1u << lane) - 1u))] = key;
        nbuf += cnt;
    }

    // Merges another top-k list, given as its ascending 32-key chunks (entry
    // 32 c + lane of the list at other[32 c + lane]), into this one (its buffer
    // empty).  Keys are unique, so the result does not depend on which list is
    // merged into which.
    __device__ __forceinline__ void merge_sorted(const unsigned long long* other, int k, int lane) {
#pragma unroll
        for (int c = 0; c < KW; ++c) {
            unsigned long long v = other[32 * c + lane];
            if (__all_sync(0xffffffffu, !(v < tau))) break;  // the rest of that list is worse
            v = v < tau ? v : ~0ull;
#pragma unroll
            for (int w = 0; w < KW; ++w) {
                const unsigned long long rc = shfl_u64(v, 31 - lane);
                const unsigned long long lo = top[w] < rc ? top[w] : rc;
                const unsigned long long hi = top[w] < rc ? rc : top[w];
                top[w] = warp_bitonic_clean(lo, lane);
                if (w + 1 < KW) {
                    if (__all_sync(0xffffffffu, hi == ~0ull)) break;
                    v = warp_bitonic_clean(hi, lane);
                }
            }
#pragma unroll
            for (int w = 0; w < KW; ++w)
                if (32 * w + lane >= k) top[w] = ~0ull;
            tau = entry(k - 1);
            tau = tau < cap ? tau : cap;
        }
    }
};

}  // namespace m3g
